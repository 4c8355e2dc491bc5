"""tl_decode_attention_static against tl_decode_attention, through the C-ABI.

tl_decode_attention_static is the decode for callers that cannot allocate
device memory when they decode — an engine whose memory all comes from its
own arena, or a path that must not risk the implicit synchronisation of
cudaMalloc/cudaFree. It reads a pool and block tables the caller owns and
keeps its split-K scratch in a fixed array inside the library, which every
call reuses. So this test makes two calls in a row with different layers
and queries (the second call starts with the first one's scratch contents)
and checks each against the handle-based entry point on the same pool and
against the CPU oracle's attention over the same logical K/V, within the
attention tolerance of the other parity tests.

The file name makes pytest collect it last, so a run that stops at the first
failure has already run every other test.
"""
import numpy as np
import pytest

import conftest
import oracle as O
import tiny_llm_b200 as T
from gpu_helpers import Run, check_close, from_dev, to_dev

pytestmark = pytest.mark.gpu


def test_static_scratch_decode_matches_handle_decode_on_two_calls():
    if not conftest.cuda_available():
        pytest.skip("no CUDA device")
    import torch

    L, Hq, Hkv, D, bs = 2, 32, 8, 128, 16
    r = Run.create(L=L, Hq=Hq, Hkv=Hkv, D=D, bs=bs, max_seq_len=5000, max_batch=6, rope=True,
                   permute_seed=9)
    lens = [4999, 1, 700, 0, 129, 2048]  # one long sequence forces many split partials
    sids = [r.allocate(5000) for _ in lens]
    for i, (sid, S) in enumerate(zip(sids, lens)):
        if S:
            r.prefill(sid, S, seed=40 + i)
    cache = r.cache

    # The caller-owned side: block tables uploaded from host copies, an error word.
    stride = cache.pool_stats().max_blocks_per_seq
    bt = np.zeros((len(sids), stride), np.int32)
    for i, sid in enumerate(sids):
        t = cache.block_table(sid)
        bt[i, : len(t)] = t
    bt_dev = torch.from_numpy(bt).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    base, _ = cache.pool()
    cfg = cache.config
    view = T.PagedView(pool=base, block_tables=bt_dev.data_ptr(), error_word=err.data_ptr(),
                       num_blocks=cfg.num_blocks, num_layers=L, num_kv_heads=Hkv, num_q_heads=Hq,
                       head_dim=D, block_size=bs, layout=cfg.layout, bt_stride=stride,
                       num_rows=len(sids))
    rows = list(range(len(sids)))
    seq_lens = [cache.get_seq_len(s) for s in sids]
    assert seq_lens == lens

    for call, layer in enumerate([0, 1]):
        qh = O.normal_f16((len(sids), Hq, D), 100 + call)
        q = to_dev(qh)
        o_ref = torch.full((len(sids), Hq, D), 0x7e00, dtype=torch.int16, device="cuda")
        cache.decode_attention(layer, q.data_ptr(), o_ref.data_ptr(), sids)
        cache.sync_check()
        o = torch.full((len(sids), Hq, D), 0x7e00, dtype=torch.int16, device="cuda")
        T.decode_attention_static(view, layer, q.data_ptr(), o.data_ptr(), rows, seq_lens)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        ref = O.f16_to_f32(from_dev(o_ref))
        got = O.f16_to_f32(from_dev(o))
        assert np.isfinite(got).all()
        check_close(got, ref, f"static-scratch call {call + 1} (layer {layer})")
        for i, sid in enumerate(sids):  # and against the oracle directly
            lk, lv = r.logical_k[(sid, layer)], r.logical_v[(sid, layer)]
            if not lk:
                assert not got[i].any(), "a sequence with no tokens must give zeros"
                continue
            want = O.decode_one(qh[i], np.stack(lk), np.stack(lv), 1.0 / np.sqrt(D))
            check_close(got[i], want, f"static-scratch call {call + 1} seq {i} vs oracle")


def test_static_scratch_rejects_oversized_requests():
    if not conftest.cuda_available():
        pytest.skip("no CUDA device")
    view = T.PagedView(pool=16, block_tables=16, error_word=None, num_blocks=4, num_layers=1,
                       num_kv_heads=1, num_q_heads=1, head_dim=128, block_size=16, layout=0,
                       bt_stride=1, num_rows=2)
    with pytest.raises(T.InvalidArgument) as e:
        T.decode_attention_static(view, 0, 16, 16, list(range(300)), [1] * 300)
    assert "num_seqs" in str(e.value)
    with pytest.raises(T.InvalidArgument) as e:  # a table row past the caller's table
        T.decode_attention_static(view, 0, 16, 16, [2], [1])
    assert "table row" in str(e.value)
    with pytest.raises(T.Unsupported):
        view.head_dim = 96
        T.decode_attention_static(view, 0, 16, 16, [0], [1])
