"""The CPU oracle against known answers and the reference's own tests.

The reference has no attention golden vectors (its attention tests only
check non-zero output and softmax row sums, tests/test_kernels.cu:436-530),
so the decode oracle is pinned here by closed-form cases, by the reference's
append round-trip test (tests/test_transformer.cu:141-194) and, in
test_golden.py, by fixtures produced by the reference's own CUDA code.
"""
import math

import numpy as np
import pytest

import oracle as O


def test_f16_to_f32_exhaustive_matches_numpy():
    bits = np.arange(65536, dtype=np.uint16)
    ours = O.f16_to_f32(bits)
    ref = bits.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(ours), nan)
    assert np.array_equal(ours[~nan].view(np.uint32), ref[~nan].view(np.uint32))


def test_f32_to_f16_round_to_nearest_even_matches_numpy():
    rng = np.random.default_rng(0)
    edge = np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e9, -1e9, 6.1035156e-05,
                     5.9604645e-08, 2.9802322e-08, 2.9802326e-08, 1.0 + 2**-11, 1.0 + 3 * 2**-11,
                     np.inf, -np.inf], dtype=np.float32)
    x = np.concatenate([edge, rng.standard_normal(200000).astype(np.float32) * 1000,
                        rng.standard_normal(200000).astype(np.float32) * 1e-6,
                        (rng.random(100000) * 2**-14).astype(np.float32)])
    ours = O.f32_to_f16(x)
    ref = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, ref)


def test_normal_generator_is_seeded_and_standard():
    a = O.normal_f16((1 << 16,), seed=7)
    b = O.normal_f16((1 << 16,), seed=7)
    c = O.normal_f16((1 << 16,), seed=8)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    f = O.f16_to_f32(a).astype(np.float64)
    assert abs(f.mean()) < 0.02 and abs(f.std() - 1.0) < 0.02


def test_rope_table_matches_documented_formula():
    cos, sin = O.rope_table(64, 128, 10000.0)
    i = np.arange(64, dtype=np.float64)
    freq = 10000.0 ** (-2.0 * i / 128)
    for pos in (0, 1, 17, 63):
        ang = pos * freq
        assert np.allclose(cos[pos], np.cos(ang), atol=1e-7)
        assert np.allclose(sin[pos], np.sin(ang), atol=1e-7)
    assert np.all(cos[0] == 1.0) and np.all(sin[0] == 0.0)


def test_rope_row_known_answers():
    cos, sin = O.rope_table(32, 64, 10000.0)
    row = O.normal_f16((4, 64), seed=3)
    # position 0 is the identity
    assert np.array_equal(O.rope_row(row, cos, sin, 0), row)
    # rotate-half: pair (i, i + D/2) is rotated by angle pos * freq_i
    pos = 13
    out = O.f16_to_f32(O.rope_row(row, cos, sin, pos)).astype(np.float64)
    x = O.f16_to_f32(row).astype(np.float64)
    c, s = cos[pos].astype(np.float64), sin[pos].astype(np.float64)
    e1 = x[:, :32] * c - x[:, 32:] * s
    e2 = x[:, 32:] * c + x[:, :32] * s
    assert np.allclose(out[:, :32], e1, atol=2e-3, rtol=1e-3)
    assert np.allclose(out[:, 32:], e2, atol=2e-3, rtol=1e-3)
    # rotation keeps each pair's norm (up to fp16 rounding)
    n_in = x[:, :32] ** 2 + x[:, 32:] ** 2
    n_out = out[:, :32] ** 2 + out[:, 32:] ** 2
    assert np.allclose(n_in, n_out, rtol=4e-3, atol=4e-3)


def test_append_round_trip_like_reference_test():
    """tests/test_transformer.cu:141-194: 4 tokens x 4 heads x 32 read back."""
    g = O.geom(num_layers=2, num_kv_heads=4, head_dim=32, block_size=16, num_blocks=8)
    pool = np.zeros(2 * 2 * 8 * 16 * 4 * 32, dtype=np.uint16)
    bt = np.array([5, 2], dtype=np.int32)
    k = O.normal_f16((4, 4, 32), seed=200)
    v = O.normal_f16((4, 4, 32), seed=201)
    O.append(pool, g, bt, layer=0, pos0=0, k=k, v=v)
    kk, vv = O.gather(pool, g, bt, 0, 4)
    assert np.array_equal(kk, k) and np.array_equal(vv, v)
    # token-major: the first block reads back contiguously as [pos][H][D]
    off = O.pool_offset(g, 0, 0, 5, 0, 0)
    assert np.array_equal(pool[off: off + k.size].reshape(k.shape), k)


@pytest.mark.parametrize("head_major", [False, True])
def test_append_crosses_blocks_and_layers(head_major):
    g = O.geom(3, 2, 64, 16, 10, head_major)
    pool = np.zeros(3 * 2 * 10 * 16 * 2 * 64, dtype=np.uint16)
    bt = np.array([7, 0, 3], dtype=np.int32)
    k = O.normal_f16((40, 2, 64), seed=1)
    v = O.normal_f16((40, 2, 64), seed=2)
    for layer in range(3):
        O.append(pool, g, bt, layer, 0, k[:25], v[:25])
        O.append(pool, g, bt, layer, 25, k[25:], v[25:])
    for layer in range(3):
        kk, vv = O.gather(pool, g, bt, layer, 40)
        assert np.array_equal(kk, k) and np.array_equal(vv, v)


def test_decode_single_token_returns_its_value():
    q = O.normal_f16((8, 64), 1)
    k = O.normal_f16((1, 2, 64), 2)
    v = O.normal_f16((1, 2, 64), 3)
    out = O.decode_one(q, k, v, 0.125)
    vf = O.f16_to_f32(v)
    for hq in range(8):
        assert np.allclose(out[hq], vf[0, hq // 4], atol=1e-6)


def test_decode_equal_keys_average_values():
    S, D = 37, 64
    q = O.normal_f16((4, D), 1)
    k = np.repeat(O.normal_f16((1, 1, D), 2), S, axis=0)
    v = O.normal_f16((S, 1, D), 3)
    out = O.decode_one(q, k, v, 1.0 / 8)
    mean = O.f16_to_f32(v)[:, 0, :].astype(np.float64).mean(axis=0)
    for hq in range(4):
        assert np.allclose(out[hq], mean, atol=1e-5)


def test_decode_dominant_key_selects_its_value():
    S, D = 50, 64
    q = O.f32_to_f16(np.full((1, D), 1.0, np.float32))
    kf = np.zeros((S, 1, D), np.float32)
    kf[17] = 4.0  # score 4*64*scale dominates
    k = O.f32_to_f16(kf)
    v = O.normal_f16((S, 1, D), 9)
    out = O.decode_one(q, k, v, 1.0)
    assert np.allclose(out[0], O.f16_to_f32(v)[17, 0], atol=1e-6)


def test_decode_matches_independent_numpy_softmax():
    S, Hq, Hkv, D = 300, 8, 2, 128
    q = O.normal_f16((Hq, D), 11)
    k = O.normal_f16((S, Hkv, D), 12)
    v = O.normal_f16((S, Hkv, D), 13)
    scale = 1.0 / math.sqrt(D)
    out = O.decode_one(q, k, v, scale)
    qf, kf, vf = (O.f16_to_f32(x).astype(np.float64) for x in (q, k, v))
    for hq in range(Hq):
        h = hq // (Hq // Hkv)
        s = kf[:, h, :] @ qf[hq] * scale
        p = np.exp(s - s.max())
        ref = (p / p.sum()) @ vf[:, h, :]
        assert np.allclose(out[hq], ref, atol=1e-6)
    # softmax rows sum to one (reference tests/test_kernels.cu:504-530)
    assert abs(p.sum() / p.sum() - 1.0) < 1e-12


def test_decode_empty_sequence_is_zero():
    q = O.normal_f16((4, 64), 1)
    out = O.decode_one(q, np.zeros((0, 1, 64), np.uint16), np.zeros((0, 1, 64), np.uint16), 0.1)
    assert np.all(out == 0)


def test_fp32_baseline_agrees_with_fp64_oracle():
    """The timed CPU baseline (reference kernel math in fp32) vs fp64."""
    Hq, Hkv, D, bs = 8, 2, 64, 16
    lens = np.array([17, 64, 100, 128], dtype=np.int32)
    nb = 40
    g = O.geom(1, Hkv, D, bs, nb)
    pool = np.zeros(2 * nb * bs * Hkv * D, dtype=np.uint16)
    rng = np.random.default_rng(0)
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.zeros((4, 8), np.int32)
    used = 0
    ks, vs = [], []
    for b, S in enumerate(lens):
        n = -(-S // bs)
        bt[b, :n] = perm[used: used + n]
        used += n
        k = O.normal_f16((S, Hkv, D), 100 + b)
        v = O.normal_f16((S, Hkv, D), 200 + b)
        O.append(pool, g, bt[b], 0, 0, k, v)
        ks.append(k)
        vs.append(v)
    q = O.normal_f16((4, Hq, D), 5)
    out, threads = O.decode_paged_f32(pool, g, 0, bt, lens, q, Hq, 0.125, threads=2)
    assert threads >= 1
    for b in range(4):
        ref = O.decode_one(q[b], ks[b], vs[b], 0.125)
        got = O.f16_to_f32(out[b])
        assert np.all(np.abs(got - ref) <= 2e-3 + 1e-3 * np.abs(ref))


@pytest.mark.parametrize("M,N,K,group", [(1, 8, 16, 16), (5, 48, 256, 32), (3, 40, 100, 8)])
def test_w8a16_matmul_against_float64(M, N, K, group):
    """The W8A16 restatement (reference kernels/w8a16_matmul.cu:71-93) is the
    product of x and the dequantised weights w * scale[k/group]: against an
    independent float64 evaluation within fp32 summation error, and exactly
    on a hand-sized case."""
    rng = np.random.default_rng(M * 100 + K)
    x = O.normal_f16((M, K), 5 + M)
    w = rng.integers(-127, 128, (K, N), dtype=np.int64).astype(np.int8)
    s = np.float16(rng.uniform(0.002, 0.02, ((K + group - 1) // group, N))).view(np.uint16)
    got = O.w8a16_matmul(x, w, s, group, threads=1).astype(np.float64)
    xf = O.f16_to_f32(x).astype(np.float64)
    wf = w.astype(np.float64) * np.repeat(O.f16_to_f32(s).astype(np.float64), group, axis=0)[:K]
    exp = xf @ wf
    bound = 1e-6 * (np.abs(xf) @ np.abs(wf)) + 1e-30
    assert (np.abs(got - exp) <= bound).all()
    # 1 x [1, 2, -3] . w (group 2: scales 0.5 then 2)
    x1 = O.f32_to_f16(np.array([[1.0, 2.0, -3.0]], np.float32))
    w1 = np.array([[4], [-5], [6]], np.int8)
    s1 = O.f32_to_f16(np.array([[0.5], [2.0]], np.float32))
    assert O.w8a16_matmul(x1, w1, s1, 2)[0, 0] == 1 * 4 * 0.5 + 2 * -5 * 0.5 + -3 * 6 * 2.0
