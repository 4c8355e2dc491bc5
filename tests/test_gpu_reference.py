"""The reference's own CUDA code (oracle/_ref, compiled unmodified from the
reference sources) as a second checker, on the same seeded inputs:

* kernels::attention_decode vs the fp64 oracle (pins the oracle to the
  reference's behaviour);
* our decode (through the C-ABI) vs kernels::attention_decode, within the
  attention tolerance |got - ref| <= 2e-3 + 1e-3|ref|;
* our append vs KVCacheManager::appendKV: getCache() read-backs byte-identical;
* kernels::w8a16_matmul vs the oracle's restatement rounded to fp16,
  bit for bit (pins that oracle), and our fused Q/K/V projection + append vs
  kernels::w8a16_matmul within two fp16 units.
"""
import math
import sys
from pathlib import Path

import numpy as np
import pytest

import conftest
import oracle as O
import tiny_llm_b200 as T
from gpu_helpers import check_close, d2h, from_dev, to_dev

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import make_golden as MG  # noqa: E402
import ref_lib  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _need():
    if not conftest.cuda_available():
        pytest.skip("no CUDA device")
    if not ref_lib.available():
        pytest.skip("oracle/_ref/libtllm_ref.so not built (needs the reference sources at build time)")


def _reference_decode(q, k, v, Hq, scale):
    import torch
    B, S, Hkv, D = k.shape
    qd = to_dev(q)
    kd, vd = to_dev(MG.expand_for_reference(k, Hq)), to_dev(MG.expand_for_reference(v, Hq))
    od = torch.zeros((B, Hq, D), dtype=torch.int16, device="cuda")
    ref_lib.attention_decode(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), od.data_ptr(), scale,
                             B, Hq, S, D)
    torch.cuda.synchronize()
    return O.f16_to_f32(from_dev(od))


@pytest.mark.parametrize("case", MG.DECODE_CASES, ids=[c[0] for c in MG.DECODE_CASES])
def test_reference_kernel_matches_oracle(case):
    name, B, Hq, Hkv, S, D, seed = case
    q, k, v = MG.decode_inputs(B, Hq, Hkv, S, D, seed)
    scale = 1.0 / math.sqrt(D)
    got = _reference_decode(q, k, v, Hq, scale)
    for b in range(B):
        ref = O.decode_one(q[b], k[b], v[b], scale, eps=1e-6)
        check_close(got[b], ref, f"reference kernel vs oracle, {name} b={b}")


@pytest.mark.parametrize("case", MG.DECODE_CASES, ids=[c[0] for c in MG.DECODE_CASES])
def test_ours_matches_reference_kernel(case):
    import torch
    name, B, Hq, Hkv, S, D, seed = case
    q, k, v = MG.decode_inputs(B, Hq, Hkv, S, D, seed)
    scale = 1.0 / math.sqrt(D)
    ref = _reference_decode(q, k, v, Hq, scale)
    cache = T.KVCache(num_layers=1, num_kv_heads=Hkv, head_dim=D, max_seq_len=S,
                      max_batch_size=B, num_q_heads=Hq)
    sids = [cache.allocate_sequence(S) for _ in range(B)]
    for b, sid in enumerate(sids):
        kd, vd = to_dev(k[b]), to_dev(v[b])
        cache.append_kv(sid, 0, kd.data_ptr(), vd.data_ptr(), S)
        cache.advance_seq_len(sid, S)
    qd = to_dev(q)
    od = torch.zeros((B, Hq, D), dtype=torch.int16, device="cuda")
    cache.decode_attention(0, qd.data_ptr(), od.data_ptr(), sids, scale)
    cache.sync_check()
    got = O.f16_to_f32(from_dev(od))
    check_close(got, ref, f"ours vs reference kernel, {name}")


def test_append_byte_identical_to_reference_manager():
    """Same append/advance sequence through both managers (the reference
    writes [pos][H][D] at current_len, kv_cache.cpp:206-233); getCache()
    read-backs must match byte for byte (ours: token-major first block)."""
    L, H, D, n = 2, 4, 32, 5
    ks = O.normal_f16((L, n, H, D), 900)
    vs = O.normal_f16((L, n, H, D), 901)
    rc = ref_lib.RefCache(L, H, D, 64, 2)
    ours = T.KVCache(num_layers=L, num_kv_heads=H, head_dim=D, max_seq_len=64, max_batch_size=2)
    rs, os_ = rc.allocate(32), ours.allocate_sequence(32)
    keep = []
    for lo, hi in ((0, 3), (3, 5)):
        for l in range(L):
            kd, vd = to_dev(ks[l, lo:hi]), to_dev(vs[l, lo:hi])
            keep += [kd, vd]
            rc.append(rs, l, kd.data_ptr(), vd.data_ptr(), hi - lo)
            ours.append_kv(os_, l, kd.data_ptr(), vd.data_ptr(), hi - lo)
        rc.advance(rs, hi - lo)
        ours.advance_seq_len(os_, hi - lo)
    ours.sync_check()
    for l in range(L):
        rk, rv = rc.get_cache(rs, l)
        ok, ov = ours.get_cache(os_, l)
        assert np.array_equal(d2h(rk, n * H * D), d2h(ok, n * H * D)), f"K layer {l}"
        assert np.array_equal(d2h(rv, n * H * D), d2h(ov, n * H * D)), f"V layer {l}"
        assert np.array_equal(d2h(ok, n * H * D).reshape(n, H, D), ks[l])
    rc.close()


@pytest.mark.parametrize("Hq,Hkv,S,D", [(8, 8, 1, 64), (4, 4, 97, 128), (8, 2, 200, 64)])
def test_prefill_matches_reference_kernel(Hq, Hkv, S, D):
    """Our paged prefill over a fresh prompt vs the reference's own
    kernels::attention_prefill on the same Q/K/V (its [B][H][S][D] layout,
    K/V repeated per query head for GQA: the reference has no grouping)."""
    import torch
    scale = 1.0 / math.sqrt(D)
    q = O.normal_f16((S, Hq, D), 71 + S)
    k = O.normal_f16((S, Hkv, D), 72 + S)
    v = O.normal_f16((S, Hkv, D), 73 + S)
    G = Hq // Hkv
    qh = np.ascontiguousarray(q.transpose(1, 0, 2))[None]  # [1][Hq][S][D]
    kh = np.ascontiguousarray(np.repeat(k, G, axis=1).transpose(1, 0, 2))[None]
    vh = np.ascontiguousarray(np.repeat(v, G, axis=1).transpose(1, 0, 2))[None]
    qd, kd, vd = to_dev(qh), to_dev(kh), to_dev(vh)
    od = torch.zeros((1, Hq, S, D), dtype=torch.int16, device="cuda")
    ref_lib.attention_prefill(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), od.data_ptr(), scale, 1, Hq, S, D)
    torch.cuda.synchronize()
    ref = O.f16_to_f32(from_dev(od)).reshape(Hq, S, D).transpose(1, 0, 2)  # [S][Hq][D]
    cache = T.KVCache(num_layers=1, num_kv_heads=Hkv, head_dim=D, max_seq_len=S,
                      max_batch_size=1, num_q_heads=Hq)
    sid = cache.allocate_sequence(S)
    kd2, vd2, qd2 = to_dev(k), to_dev(v), to_dev(q)
    cache.append_kv(sid, 0, kd2.data_ptr(), vd2.data_ptr(), S)
    o2 = torch.zeros((S, Hq, D), dtype=torch.int16, device="cuda")
    cache.prefill_attention(0, qd2.data_ptr(), o2.data_ptr(), [sid], [S], scale)
    cache.sync_check()
    got = O.f16_to_f32(from_dev(o2)).reshape(S, Hq, D)
    check_close(got, ref, f"prefill ours vs reference kernel S={S} Hq={Hq} Hkv={Hkv}")


def _w8a16_case(M, N, K, group, seed):
    rng = np.random.default_rng(seed)
    x = O.normal_f16((M, K), seed)
    w = rng.integers(-127, 128, (K, N), dtype=np.int64).astype(np.int8)
    s = np.float16(rng.uniform(0.002, 0.02, ((K + group - 1) // group, N))).view(np.uint16)
    return x, w, s


def _reference_w8a16(x, w, s, group):
    import torch
    M, K = x.shape
    N = w.shape[1]
    xd, sd = to_dev(x), to_dev(s)
    wd = torch.from_numpy(w.copy()).cuda()
    od = torch.zeros((M, N), dtype=torch.int16, device="cuda")
    ref_lib.w8a16_matmul(xd.data_ptr(), wd.data_ptr(), sd.data_ptr(), od.data_ptr(), M, N, K, group)
    torch.cuda.synchronize()
    return from_dev(od)


@pytest.mark.parametrize("M,N,K,group", [(1, 256, 512, 32), (5, 128, 256, 16), (33, 384, 1024, 128),
                                         (64, 256, 384, 64), (3, 40, 100, 8)])
def test_oracle_w8a16_matches_reference_kernel(M, N, K, group):
    """kernels::w8a16_matmul (its reference kernel when M*N < 4096, the tiled
    one otherwise) equals the oracle's fp32 restatement rounded to fp16, bit
    for bit."""
    x, w, s = _w8a16_case(M, N, K, group, 11 + M)
    got = _reference_w8a16(x, w, s, group)
    exp = O.f32_to_f16(O.w8a16_matmul(x, w, s, group))
    assert np.array_equal(got, exp), f"{int((got != exp).sum())} of {got.size} differ"


@pytest.mark.parametrize("B,hidden,group", [(1, 512, 32), (32, 1024, 128)])
def test_projection_matches_reference_kernel(B, hidden, group):
    """Our fused projection (no RoPE) writes the same K/V rows, within two
    fp16 units, as kernels::w8a16_matmul produces for k_buf_/v_buf_."""
    import torch
    Hkv, G, D, bs, L = 2, 4, 128, 16, 2
    cache = T.KVCache(num_layers=L, num_kv_heads=Hkv, head_dim=D, max_seq_len=64, max_batch_size=B,
                      block_size=bs, num_q_heads=Hkv * G)
    sids = [cache.allocate_sequence(64) for _ in range(B)]
    x, wq, sq = _w8a16_case(B, Hkv * G * D, hidden, group, 21)
    _, wk, sk = _w8a16_case(B, Hkv * D, hidden, group, 22)
    _, wv, sv = _w8a16_case(B, Hkv * D, hidden, group, 23)
    dev = [to_dev(a) if a.dtype == np.uint16 else torch.from_numpy(a.copy()).cuda() for a in
           (x, wq, sq, wk, sk, wv, sv)]
    qd = torch.zeros((B, Hkv * G * D), dtype=torch.int16, device="cuda")
    cache.project_qkv_append(0, dev[0].data_ptr(), hidden, dev[1].data_ptr(), dev[2].data_ptr(),
                             dev[3].data_ptr(), dev[4].data_ptr(), dev[5].data_ptr(), dev[6].data_ptr(), group,
                             sids, qd.data_ptr())
    cache.sync_check()
    ref = {name: O.f16_to_f32(_reference_w8a16(x, w, s, group)).astype(np.float64)
           for name, w, s in (("q", wq, sq), ("k", wk, sk), ("v", wv, sv))}
    got_q = O.f16_to_f32(from_dev(qd)).astype(np.float64)
    base, n = cache.pool()
    pool = d2h(base, n)
    g = O.geom(L, Hkv, D, bs, cache.config.num_blocks)

    rows_k, rows_v = [], []
    for sid in sids:
        bt = np.array(cache.block_table(sid), np.int32)
        k, v = O.gather(pool, g, bt, 0, 1)
        rows_k.append(O.f16_to_f32(k[0]).reshape(-1))
        rows_v.append(O.f16_to_f32(v[0]).reshape(-1))
    for name, got in (("q", got_q), ("k", np.stack(rows_k)), ("v", np.stack(rows_v))):
        exp = ref[name]
        tol = 2.0 ** (np.floor(np.log2(np.abs(exp).max(axis=1, keepdims=True) + 1e-30)) - 9)
        assert not (np.abs(got - exp) > tol).any(), f"{name}: max err {np.abs(got - exp).max():.3e}"
