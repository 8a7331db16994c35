"""Barrier protocol of the CTA-pair GEMM (csrc/gemm_pair.cu), checked on a host
model (no GPU). Two CTAs, even (E) and odd (O), share a ring of S stages:

* both producers fill stage i % S for K-step i: from i >= S on, each first
  waits its OWN empty barrier for the phase that the MMA of step i - S
  completes; E's producer arrives on E's full barrier expecting both CTAs'
  bytes; both CTAs' TMA loads (of random latency) count their bytes on E's
  full barrier and land in their own CTA's stage;
* E's MMA thread waits E's full barrier for step i's phase, runs the MMA (it
  reads stage i % S of BOTH CTAs), and its commit arrives, when the MMA is
  done, on the empty barrier of both CTAs, then on both accumulator barriers;
* each producer finally waits the phases of its last min(S, steps) empty
  arrivals, each epilogue waits its accumulator barrier.

The model follows mbarrier semantics (a phase completes when the pending
arrivals and the transaction count reach zero; the count may go negative
first; a parity wait passes once that phase has completed), runs random
interleavings, and checks: nothing deadlocks; every MMA reads step i's data
in both CTAs; no TMA load overwrites a stage an earlier MMA still needs;
nothing is still in flight towards a CTA when it reaches its exit."""
import random


class Barrier:
    def __init__(self, count):
        self.count, self.pending, self.tx, self.phase = count, count, 0, 0

    def _maybe_complete(self):
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count

    def arrive(self, expect_tx=0):
        self.tx += expect_tx
        self.pending -= 1
        assert self.pending >= 0
        self._maybe_complete()

    def complete_tx(self, nbytes):
        self.tx -= nbytes
        self._maybe_complete()

    def passed(self, parity):  # try_wait.parity: the phase with this parity has completed
        return (self.phase & 1) != parity


def _run(nkb, S, seed, stage_bytes=10, skip_empty_wait=False):
    rng = random.Random(seed)
    full = [Barrier(1) for _ in range(S)]            # even CTA only
    empty = {c: [Barrier(1) for _ in range(S)] for c in "EO"}
    acc = {c: Barrier(1) for c in "EO"}
    stage_data = {c: [None] * S for c in "EO"}      # which K-step's data each stage holds
    mma_done = [False] * nkb
    inflight = []                                     # pending async events: (kind, payload)
    # actor states
    prod = {c: {"i": 0, "phase": "fill", "tail": max(0, nkb - S)} for c in "EO"}
    mma = {"i": 0, "state": "wait", "acc_committed": False}
    epi = {c: False for c in "EO"}

    def producer_step(c):
        st = prod[c]
        if st["phase"] == "fill":
            i = st["i"]
            if i == nkb:
                st["phase"] = "tail"
                return True
            s = i % S
            if i >= S and not skip_empty_wait and not empty[c][s].passed(((i // S) - 1) & 1):
                return False
            if c == "E":
                full[s].arrive(expect_tx=2 * stage_bytes)
            inflight.append(("tma", (c, i)))
            st["i"] += 1
            return True
        if st["phase"] == "tail":
            i = st["tail"]
            if i >= nkb:
                st["phase"] = "done"
                return True
            if not empty[c][i % S].passed((i // S) & 1):
                return False
            st["tail"] += 1
            return True
        return False

    def mma_step():
        i = mma["i"]
        if i == nkb:
            if not mma["acc_committed"]:
                inflight.append(("commit_acc", None))
                mma["acc_committed"] = True
                return True
            return False
        s = i % S
        if not full[s].passed((i // S) & 1):
            return False
        # the MMA reads stage s of both CTAs: both must hold step i's data
        assert stage_data["E"][s] == i and stage_data["O"][s] == i, (i, stage_data)
        inflight.append(("mma", i))
        mma["i"] += 1
        return True

    def deliver(ev):
        kind, payload = ev
        if kind == "tma":
            c, i = payload
            s = i % S
            # the stage may only be overwritten once the MMA of step i - S is done
            assert i < S or mma_done[i - S], ("TMA overwrote a stage still in use", c, i)
            stage_data[c][s] = i
            full[s].complete_tx(stage_bytes)
        elif kind == "mma":
            i = payload
            mma_done[i] = True
            for c in "EO":
                empty[c][i % S].arrive()
        elif kind == "commit_acc":
            assert all(mma_done)
            for c in "EO":
                acc[c].arrive()

    for _ in range(200000):
        actions = []
        for c in "EO":
            if prod[c]["phase"] != "done":
                actions.append(("prod", c))
            if not epi[c]:
                actions.append(("epi", c))
        if not mma["acc_committed"]:
            actions.append(("mma", None))
        if inflight:
            actions.append(("deliver", None))
        if not actions:
            break
        kind, c = rng.choice(actions)
        if kind == "prod":
            producer_step(c)
        elif kind == "mma":
            mma_step()
        elif kind == "epi":
            if acc[c].passed(0):
                epi[c] = True
        else:  # MMAs (and the commit after them) complete in issue order; loads in any order
            mmas = [e for e in inflight if e[0] in ("mma", "commit_acc")]
            loads = [e for e in inflight if e[0] == "tma"]
            pick = rng.choice(([mmas[0]] if mmas else []) + loads)
            inflight.remove(pick)
            deliver(pick)
        if all(p["phase"] == "done" for p in prod.values()) and all(epi.values()):
            # both CTAs are at their final cluster barrier and exit: nothing may still be on its way
            assert not inflight, inflight
    else:
        return False
    # exit: both producers and epilogues finished, nothing in flight towards either CTA
    assert all(p["phase"] == "done" for p in prod.values()) and all(epi.values()) and not inflight
    return True


def test_pair_protocol_never_deadlocks_or_races():
    for nkb in (1, 2, 5, 6, 7, 13, 22, 64):
        for S in (4, 6, 8):
            for seed in range(8):
                assert _run(nkb, S, seed), (nkb, S, seed)


def test_model_catches_a_producer_that_skips_its_empty_wait():
    """The checks have teeth: producers that do not wait for the stage
    release overwrite a stage the MMA still needs."""
    caught = 0
    for seed in range(20):
        try:
            _run(9, 4, seed, skip_empty_wait=True)
        except AssertionError:
            caught += 1
    assert caught > 0
