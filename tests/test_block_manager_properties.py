"""Property test of the block allocator (hypothesis, CPU): random streams of
prompt allocations (with shared prefixes, so the prefix cache hits),
decode-step growth and frees keep the pool consistent after every operation:
every block is either free or in use, never both; reference counts equal the
number of live block tables that hold the block; every cache key points to a
block that carries that key; a sequence's cached prefix holds exactly the
tokens of its first blocks."""
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from kavor_b200.engine.block_manager import BlockManager

BS = 4
POOL = 24
PREFIXES = [list(range(100, 100 + 3 * BS)), list(range(200, 200 + 2 * BS)), [7] * (2 * BS)]


def _check(bm: BlockManager, live) -> None:
    free, used = set(bm.free_block_ids), bm.used_block_ids
    assert not free & used and len(free) + len(used) == POOL and len(free) == len(bm.free_block_ids)
    refs = {}
    for s in live:
        for b in s.block_table:
            refs[b] = refs.get(b, 0) + 1
    assert set(refs) == used
    for b, n in refs.items():
        assert bm.blocks[b].ref_count == n
    for key, b in bm.hash_to_block_id.items():
        assert bm.blocks[b].hash == key
    for s in live:
        for i in range(s.num_cached_tokens // BS):
            if bm.blocks[s.block_table[i]].hash != -1:
                assert bm.blocks[s.block_table[i]].token_ids == s.block(i)


ops = st.lists(st.tuples(st.sampled_from(["add", "add", "grow", "free"]), st.integers(0, 10_000)),
               min_size=1, max_size=40)


@settings(max_examples=150, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])  # stateless factory
@given(ops)
def test_pool_stays_consistent(make_seq, program):
    bm = BlockManager(POOL, BS)
    live = []
    for op, k in program:
        if op == "add":
            prefix = PREFIXES[k % len(PREFIXES)]
            tail = [k % 97 + 1000 + j for j in range(k % (2 * BS) + 1)]
            s = make_seq(prefix + tail)
            cached, _ = bm.can_allocate_prefill(s)
            if cached == -1:
                continue
            bm.allocate_prefill(s, cached)
            # the whole prompt runs in one step; its full blocks get keyed
            s.num_scheduled_tokens = len(s) - s.num_cached_tokens
            bm.hash_blocks(s)
            s.num_cached_tokens = len(s)
            s.num_scheduled_tokens = 0
            live.append(s)
        elif op == "grow" and live:
            s = live[k % len(live)]
            s.append_token(k % 50)
            if not bm.can_append_block(s):
                s.num_tokens -= 1
                s.token_ids.pop()
                s.last_token = s.token_ids[-1]
                continue
            bm.may_append_block(s)
            s.num_cached_tokens = len(s) - 1
        elif op == "free" and live:
            bm.deallocate(live.pop(k % len(live)))
        _check(bm, live)
    for s in live:
        bm.deallocate(s)
    _check(bm, [])
    assert len(bm.free_block_ids) == POOL


@settings(max_examples=50, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(st.lists(st.integers(1, 3 * BS), min_size=1, max_size=5), st.integers(1, 2 * BS))
def test_batched_may_append_equals_the_per_sequence_call(make_seq, lengths, steps):
    """may_append_blocks(batch) takes the same blocks, in the same order, as
    may_append_block over the batch, step after step."""
    pools = [BlockManager(POOL * 8, BS, enable_prefix_cache=False) for _ in range(2)]
    batches = [[make_seq(range(n)) for n in lengths] for _ in range(2)]
    for bm, seqs in zip(pools, batches):
        for s in seqs:
            bm.allocate_prefill(s, 0)
    for _ in range(steps):
        for s in batches[0]:
            pools[0].may_append_block(s)
        pools[1].may_append_blocks(batches[1])
        assert [s.block_table for s in batches[0]] == [s.block_table for s in batches[1]]
        for seqs in batches:
            for s in seqs:
                s.append_token(0)
    assert pools[0].free_block_ids == pools[1].free_block_ids
