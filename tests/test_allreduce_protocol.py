"""Arrival protocol of the fused all-reduce's NVLink SHARP modes, checked on a
host model (no GPU): W ranks run the same sequence of calls, each call in
switch one-shot (one arrival round) or two-shot (two rounds) over a varying
number of blocks; a round is `multimem.red` +1 on the block's counter word at
every rank, then a wait until this rank's copy reaches W x (the block's calls
that used that word). The model interleaves the ranks at random (a rank may
run ahead into later calls as long as it never passes a wait early) and checks
that no wait ever completes before every rank has arrived at that round, and
that every wait completes (no rank is left waiting on a count that can never
be reached) — including a one-shot call followed by a two-shot call, where a
single counter shared by both words would leave the second word behind. This
is the rule `ar_add_rmsnorm_kernel` (csrc/allreduce.cu) implements with one
call counter per word."""
import random

W = 8
MAX_BLOCKS = 256


class Rank:
    def __init__(self):
        self.calls = {0: [0] * MAX_BLOCKS, 1: [0] * MAX_BLOCKS}  # per word: calls that used it, per block


def _run(program, per_word_counters, seed):
    """program: list of (mode, blocks); mode 1 = one-shot (word 0), 2 = two-shot (words 0 and 1)."""
    rng = random.Random(seed)
    words = [[[0] * MAX_BLOCKS for _ in range(2)] for _ in range(W)]  # each rank's copy of the counter words
    ranks = [Rank() for _ in range(W)]
    # per rank: position = (call index, block, round); a rank runs its blocks round by round
    state = [dict(call=0, stage="arrive", rnd=0, targets={}) for _ in range(W)]
    arrivals = {}  # (call, block, round) -> number of ranks arrived
    steps = 0
    while True:
        active = [r for r in range(W) if state[r]["call"] < len(program)]
        if not active:
            return True
        r = rng.choice(active)
        st = state[r]
        mode, blocks = program[st["call"]]
        rounds = 1 if mode == 1 else 2
        if st["stage"] == "arrive":
            for b in range(blocks):  # all blocks of the call arrive at this round
                word = st["rnd"]
                if per_word_counters:
                    ranks[r].calls[word][b] += 1
                    v = ranks[r].calls[word][b]
                else:  # one counter for both words: counts calls, not uses of the word
                    if st["rnd"] == 0:
                        ranks[r].calls[0][b] += 1
                    v = ranks[r].calls[0][b]
                st["targets"][b] = W * v
                for q in range(W):  # the switch adds 1 to every rank's copy
                    words[q][word][b] += 1
                arrivals[(st["call"], b, st["rnd"])] = arrivals.get((st["call"], b, st["rnd"]), 0) + 1
            st["stage"] = "wait"
        else:
            word = st["rnd"]
            if all(words[r][word][b] >= st["targets"][b] for b in range(blocks)):
                for b in range(blocks):  # a wait that completes must not be early
                    assert arrivals[(st["call"], b, st["rnd"])] == W, "a wait passed before every rank arrived"
                st["rnd"] += 1
                st["stage"] = "arrive"
                if st["rnd"] == rounds:
                    st.update(call=st["call"] + 1, rnd=0, targets={})
        steps += 1
        if steps > 200000:
            return False  # some rank waits on a count that is never reached


def _program(seed):
    rng = random.Random(seed)
    return [(rng.choice((1, 2)), rng.choice((1, 7, 32, 125, 256))) for _ in range(12)] + [(1, 16), (2, 16)]


def test_per_word_counters_never_release_early_and_always_complete():
    for seed in range(20):
        assert _run(_program(seed), per_word_counters=True, seed=seed)


def test_a_shared_counter_stalls_a_two_shot_after_a_one_shot():
    assert not _run([(1, 4), (2, 4)], per_word_counters=False, seed=0)
