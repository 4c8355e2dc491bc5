"""Continuous-batching churn on the GPU, checked against the oracle (config 5's
behaviour at a size the fp64 oracle can follow).

The seeded schedule of tiny_llm_b200.churn (Poisson arrivals, log-uniform
prompts, geometric generations, admission under an occupancy watermark,
recompute-style preemption, release on completion) drives a small pool held
near 80 % occupancy for 200 steps. releaseSequence (reference
src/kv_cache.cpp:121-137) returns blocks to a LIFO free list, so new
sequences take blocks — often partly written ones — that still hold a dead
sequence's K/V, and appendKV (src/kv_cache.cpp:168-238) writes at each new
sequence's current length over them. Every few steps the test checks:
  * every live sequence's K/V gathered from the device pool through its block
    table equals the oracle's logical copy bit for bit (RoPE on K), so no
    stale row is read as data and no write landed in another sequence's block;
  * decode attention of every layer over the live batch equals the fp64
    oracle within |got - ref| <= 2e-3 + 1e-3|ref| — stale rows past each
    sequence's length never reach the softmax.
"""
import numpy as np
import pytest

import conftest
from gpu_helpers import Run

pytestmark = pytest.mark.gpu


class _Tracked:
    """The cache as the churn schedule sees it, with the oracle's logical
    K/V kept in step: allocation opens a logical sequence, release drops it
    and records the blocks it gave back."""

    def __init__(self, run: Run):
        self.run = run
        self.cache = run.cache
        self.released_blocks: set[int] = set()
        self.reused = 0  # later sequences that took at least one released block

    def allocate_sequence(self, max_len):
        sid = self.run.allocate(max_len)
        if set(self.cache.block_table(sid)) & self.released_blocks:
            self.reused += 1
        return sid

    def release_sequence(self, sid):
        self.released_blocks.update(self.cache.block_table(sid))
        self.cache.release_sequence(sid)
        self.run.seqs.remove(sid)
        for l in range(self.run.L):
            del self.run.logical_k[(sid, l)]
            del self.run.logical_v[(sid, l)]

    def pool_stats(self):
        return self.cache.pool_stats()

    def get_seq_len(self, sid):
        return self.cache.get_seq_len(sid)


@pytest.mark.parametrize("layout", ["token", "head"])
def test_churn_release_reuse_matches_oracle(layout):
    if not conftest.cuda_available():
        pytest.skip("no CUDA device")
    import tiny_llm_b200 as T
    from tiny_llm_b200.churn import ChurnSchedule

    L, Hq, Hkv, D, bs = 2, 16, 4, 128, 16
    max_active, lo, hi, gen_mean, max_len = 24, 8, 300, 24, 512
    nblocks = ChurnSchedule.pool_blocks_for(max_active, lo, hi, gen_mean, bs, occupancy=0.8)
    r = Run.create(L=L, Hq=Hq, Hkv=Hkv, D=D, bs=bs, max_seq_len=max_len, max_batch=max_active,
                   rope=True, num_blocks=nblocks, permute_seed=3,
                   layout=T.TL_LAYOUT_HEAD_MAJOR if layout == "head" else T.TL_LAYOUT_TOKEN_MAJOR)
    tracked = _Tracked(r)
    sch = ChurnSchedule(seed=11, rate=1.5, prompt_lo=lo, prompt_hi=hi, gen_mean=gen_mean,
                        max_active=max_active, block_size=bs, occupancy_target=0.8)
    counter = [0]

    def prefill(sid, n):
        counter[0] += 1
        r.prefill(sid, n, seed=10_000 + counter[0])

    step_no = [0]
    checked = [0]

    def decode_step(batch):
        i = step_no[0]
        r.step_append(batch, seed=500_000 + 2 * i)
        if i % 4 == 0 or i >= 190:
            for l in range(L):
                r.decode_and_check(l, batch, seed=900_000 + 10 * i + l)
            checked[0] += 1
        if i % 20 == 0:
            r.check_pool_bit_exact()
        for s in batch:
            r.cache.advance_seq_len(s, 1)

    occ = []
    for i in range(200):
        step_no[0] = i
        sch.step(tracked, prefill, decode_step, max_len)
        st = r.cache.pool_stats()
        occ.append(st.used_blocks / st.num_blocks)
    r.cache.sync_check()
    r.check_pool_bit_exact()

    s = sch.stats
    assert s.released >= 20, f"only {s.released} releases in 200 steps"
    assert tracked.reused >= 10, f"only {tracked.reused} sequences took released blocks"
    assert checked[0] >= 50
    assert np.mean(occ[50:]) > 0.6, f"pool not held near its target: {np.mean(occ[50:]):.2f}"
    assert r.cache.pool_stats().used_blocks + r.cache.pool_stats().free_blocks == nblocks
