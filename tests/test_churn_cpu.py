"""The churn schedule (config 5's continuous batching) on the bookkeeping
backend: the block allocator keeps exact accounting through thousands of
allocate / grow / release events, never leaks, and holds occupancy near the
pool-sizing target."""
import tiny_llm_b200 as T
from tiny_llm_b200.churn import ChurnSchedule


def test_churn_block_accounting_and_no_leaks():
    bs, max_active = 16, 64
    nblocks = ChurnSchedule.pool_blocks_for(max_active, 32, 4096, 256, bs, occupancy=0.8)
    cache = T.KVCache(num_layers=2, num_kv_heads=2, head_dim=64, max_seq_len=6144,
                      max_batch_size=max_active, block_size=bs, num_blocks=nblocks,
                      backend=T.TL_BACKEND_HOST_BOOKKEEPING)
    cache.permute_free_blocks(3)
    sch = ChurnSchedule(seed=5, rate=4.0, max_active=max_active, block_size=bs)

    def prefill(sid, n):
        cache.reserve(sid, n)
        cache.advance_seq_len(sid, n)

    def decode_step(batch):
        for s in batch:
            cache.reserve(s, cache.get_seq_len(s) + 1)  # the appended token's block
            cache.advance_seq_len(s, 1)

    for _ in range(600):
        sch.step(cache, prefill, decode_step, max_len=6144)
        st = cache.pool_stats()
        expect = sum(-(-cache.get_seq_len(r.seq_id) // bs) for r in sch.active)
        assert st.used_blocks == expect
        assert st.used_blocks + st.free_blocks == st.num_blocks
        assert st.active_sequences == len(sch.active) <= max_active
    s = sch.stats
    assert s.admitted > 150 and s.released > 100 and s.max_active == max_active
    assert 0.5 < s.occupancy_sum / s.steps < 0.95
    for r in list(sch.active):
        cache.release_sequence(r.seq_id)
    st = cache.pool_stats()
    assert st.used_blocks == 0 and st.free_blocks == st.num_blocks
