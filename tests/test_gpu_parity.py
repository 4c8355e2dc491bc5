"""Parity of the CUDA path (through the C-ABI) with the CPU oracle.

Append / block-table gathers: bit-exact. Decode attention: elementwise
|got - ref| <= 2e-3 + 1e-3*|ref| against the fp64 restatement of the
reference kernel's math (kernels/attention.cu:34-111) generalised to GQA.
"""
import math

import numpy as np
import pytest

import conftest
import oracle as O
import tiny_llm_b200 as T
from gpu_helpers import Run, check_close, d2h, from_dev, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _need_gpu():
    if not conftest.cuda_available():
        pytest.skip("no CUDA device")


@pytest.mark.parametrize("rope", [False, True])
@pytest.mark.parametrize("layout", [T.TL_LAYOUT_TOKEN_MAJOR, T.TL_LAYOUT_HEAD_MAJOR])
def test_config1_tiny_gqa_end_to_end(rope, layout):
    """L=2, Hq=8, Hkv=2, D=64, bs=16, prompts {17,64,100,128},
    then 32 decode steps (fused append + decode per layer + advance)."""
    r = Run.create(L=2, Hq=8, Hkv=2, D=64, bs=16, max_seq_len=256, max_batch=4, rope=rope,
                   layout=layout)
    prompts = [17, 64, 100, 128]
    sids = [r.allocate(P + 32) for P in prompts]
    for i, (sid, P) in enumerate(zip(sids, prompts)):
        r.prefill(sid, P, seed=10 + i)
    r.check_pool_bit_exact()
    for step in range(32):
        r.step_append(sids, seed=5000 + 7 * step)
        for layer in range(2):
            r.decode_and_check(layer, sids, seed=9000 + 3 * step + layer)
        for sid in sids:
            r.cache.advance_seq_len(sid, 1)
    r.check_pool_bit_exact()
    for sid, P in zip(sids, prompts):
        assert r.cache.get_seq_len(sid) == P + 32


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("G", [1, 4, 8])
@pytest.mark.parametrize("bs", [16, 32])
def test_decode_shapes(D, G, bs):
    Hkv = 2
    r = Run.create(L=1, Hq=Hkv * G, Hkv=Hkv, D=D, bs=bs, max_seq_len=700, max_batch=5,
                   rope=(G == 4), permute_seed=3)
    lens = [1, 16, 33, 300, 640]
    sids = [r.allocate(700) for _ in lens]
    for i, (sid, S) in enumerate(zip(sids, lens)):
        r.prefill(sid, S, seed=100 + i)
    r.check_pool_bit_exact()
    r.decode_and_check(0, sids, seed=77)


@pytest.mark.parametrize("D,G,rope,bs", [(128, 4, True, 16), (64, 8, True, 32), (256, 1, True, 16),
                                         (128, 8, False, 32)])
def test_attention_step_engine_flow(D, G, rope, bs):
    """The decode branch of TransformerLayer::attention for a batch, layer by
    layer (per-layer append of the new token, then decode with RoPE on Q at
    the same position), over several steps of ragged sequences; the pool
    stays bit-exact."""
    Hkv = 2
    r = Run.create(L=2, Hq=Hkv * G, Hkv=Hkv, D=D, bs=bs, max_seq_len=600, max_batch=6, rope=rope,
                   permute_seed=11)
    # new tokens land mid-tile, at the start of a tile (built without a load)
    # and at the start of a block (a block the kernel enters in the table)
    lens = [1, 15, 16, 47, 300, 511]
    sids = [r.allocate(600) for _ in lens]
    for i, (sid, S) in enumerate(zip(sids, lens)):
        r.prefill(sid, S, seed=400 + i)
    for step in range(4):
        for layer in range(2):
            r.attention_step_and_check(layer, sids, seed=7000 + 10 * step + 3 * layer)
        for sid in sids:
            r.cache.advance_seq_len(sid, 1)
    r.check_pool_bit_exact()
    for sid, S in zip(sids, lens):
        assert r.cache.get_seq_len(sid) == S + 4


def test_attention_step_overwrites_pending_token_and_refuses_unadvanced_runs():
    """One token appended at the current length and not advanced is
    overwritten by the step (same position); a multi-token run appended past
    the length and not advanced is refused before any state changes."""
    r = Run.create(L=1, Hq=8, Hkv=2, D=128, bs=16, max_seq_len=200, max_batch=2, rope=True)
    sids = [r.allocate(200) for _ in range(2)]
    for i, sid in enumerate(sids):
        r.prefill(sid, 40 + i, seed=800 + i)
    r.step_append(sids, seed=810)                  # position len, pending
    r.attention_step_and_check(0, sids, seed=820)  # the same position again
    r.check_pool_bit_exact()
    for sid in sids:
        r.cache.advance_seq_len(sid, 1)
    k = O.normal_f16((2, r.Hkv, r.D), 830)
    kd = to_dev(k)
    r.cache.append_kv(sids[0], 0, kd.data_ptr(), kd.data_ptr(), 2)  # two pending tokens
    used = r.cache.pool_stats().used_blocks
    with pytest.raises(T.InvalidArgument) as e:
        r.cache.attention_step(0, kd.data_ptr(), kd.data_ptr(), kd.data_ptr(), kd.data_ptr(), sids)
    assert "advance it first" in str(e.value)
    assert r.cache.pool_stats().used_blocks == used


def _prefill_and_check(r, sids, prefixes, ntoks, seed):
    """Appends ntoks[i] prompt tokens after a cached prefix of prefixes[i]
    tokens, runs the paged prefill over them and checks every query row
    against the oracle: the fp64 decode restatement over the tokens up to
    the row's position (Q rotated at that position when K is)."""
    import torch
    for i, (sid, P0, n) in enumerate(zip(sids, prefixes, ntoks)):
        if P0:
            r.prefill(sid, P0, seed=seed + 10 * i)  # appended and advanced
        k = O.normal_f16((n, r.Hkv, r.D), seed + 10 * i + 1)
        v = O.normal_f16((n, r.Hkv, r.D), seed + 10 * i + 2)
        kd, vd = to_dev(k), to_dev(v)
        r.cache.append_kv(sid, 0, kd.data_ptr(), vd.data_ptr(), n)
        r._record(sid, 0, P0, k, v)
    rows = sum(ntoks)
    q = O.normal_f16((rows, r.Hq, r.D), seed + 999)
    qd = to_dev(q)
    od = torch.full((rows, r.Hq, r.D), 0x7e00, dtype=torch.int16, device="cuda")  # NaN fill
    sc = 1.0 / math.sqrt(r.D)
    r.cache.prefill_attention(0, qd.data_ptr(), od.data_ptr(), sids, ntoks, sc)
    r.cache.sync_check()
    got = O.f16_to_f32(from_dev(od))
    row = 0
    for sid, P0, n in zip(sids, prefixes, ntoks):
        kk = np.stack(r.logical_k[(sid, 0)])
        vv = np.stack(r.logical_v[(sid, 0)])
        for j in range(n):
            pos = P0 + j
            qj = O.rope_row(q[row], r.cos, r.sin, pos) if r.rope else q[row]
            ref = O.decode_one(qj, kk[:pos + 1], vv[:pos + 1], sc)
            check_close(got[row], ref, f"prefill seq {sid} row {j} pos {pos}")
            row += 1


@pytest.mark.parametrize("D,G,bs,rope", [(128, 1, 16, True), (128, 4, 32, True), (64, 8, 16, False),
                                         (128, 3, 16, True), (64, 2, 32, True)])
def test_prefill_attention_over_cached_prefix(D, G, bs, rope):
    """Paged causal prefill (replacing kernels::attention_prefill): prompts
    of several lengths (one token to several CTAs of query rows), alone and
    after a cached prefix, in one call; the grouped query heads (G = 3 is
    padded to 4 in the CTA's rows) share their KV head."""
    Hkv = 2
    r = Run.create(L=1, Hq=Hkv * G, Hkv=Hkv, D=D, bs=bs, max_seq_len=400, max_batch=5, rope=rope,
                   permute_seed=17)
    prefixes = [0, 0, 5, 100, 33]
    ntoks = [1, 130, 17, 64, 200]
    sids = [r.allocate(400) for _ in prefixes]
    _prefill_and_check(r, sids, prefixes, ntoks, seed=1234 + D + G)
    r.check_pool_bit_exact()


def test_single_long_sequence_many_splits():
    """One KV head, one long sequence: every worker gets a slice of the same
    unit, so the merge pass combines hundreds of partials."""
    r = Run.create(L=1, Hq=8, Hkv=1, D=128, bs=16, max_seq_len=9000, max_batch=1)
    sid = r.allocate(9000)
    r.prefill(sid, 8999, seed=5)
    r.decode_and_check(0, [sid], seed=6)


def test_ragged_permuted_batch_and_subsets():
    r = Run.create(L=2, Hq=32, Hkv=8, D=128, bs=16, max_seq_len=1200, max_batch=12,
                   permute_seed=42)
    rng = np.random.default_rng(0)
    lens = rng.integers(1, 1100, size=12)
    sids = [r.allocate(1200) for _ in lens]
    for i, (sid, S) in enumerate(zip(sids, lens)):
        r.prefill(sid, int(S), seed=300 + i)
    r.check_pool_bit_exact()
    r.decode_and_check(1, sids, seed=1)
    r.decode_and_check(0, sids[::3], seed=2)            # a subset, out of order
    r.decode_and_check(0, [sids[5], sids[5]], seed=3)   # duplicates are fine for decode


def test_empty_sequence_decodes_to_zero_and_others_unaffected():
    r = Run.create(L=1, Hq=4, Hkv=1, D=64, bs=16, max_seq_len=64, max_batch=3)
    a = r.allocate(64)
    b = r.allocate(64)
    r.prefill(b, 20, seed=1)
    r.decode_and_check(0, [a, b], seed=2)


def test_append_then_decode_sees_pending_token():
    """Reference decode semantics (src/transformer.cpp:230-237): after
    appendKV and before advanceSeqLen the decode covers getSeqLen()+1."""
    r = Run.create(L=1, Hq=8, Hkv=2, D=64, bs=16, max_seq_len=64, max_batch=1)
    s = r.allocate(64)
    r.prefill(s, 16, seed=1)
    k = O.normal_f16((1, 2, 64), 50)
    v = O.normal_f16((1, 2, 64), 51)
    kd, vd = to_dev(k), to_dev(v)
    r.cache.append_kv(s, 0, kd.data_ptr(), vd.data_ptr(), 1)
    r._record(s, 0, 16, k, v)
    assert r.cache.get_seq_len(s) == 16
    r.decode_and_check(0, [s], seed=3)  # attends 17 tokens
    r.cache.advance_seq_len(s, 1)
    assert r.cache.get_seq_len(s) == 17


def test_reference_append_retrieve_contiguous_get_cache():
    """tests/test_transformer.cu:141-194: 4 tokens x 4 heads x 32 read back
    contiguously from the getCache pointer (token-major first block)."""
    c = T.KVCache(num_layers=2, num_kv_heads=4, head_dim=32, max_seq_len=64, max_batch_size=2)
    s = c.allocate_sequence(32)
    k = O.normal_f16((4, 4, 32), 200)
    v = O.normal_f16((4, 4, 32), 201)
    kd, vd = to_dev(k), to_dev(v)
    c.append_kv(s, 0, kd.data_ptr(), vd.data_ptr(), 4)
    c.sync_check()
    assert c.get_seq_len(s) == 0
    c.advance_seq_len(s, 4)
    assert c.get_seq_len(s) == 4
    kp, vp = c.get_cache(s, 0)
    assert np.array_equal(d2h(kp, k.size).reshape(k.shape), k)
    assert np.array_equal(d2h(vp, v.size).reshape(v.shape), v)


def test_block_exhaustion_on_device_keeps_state():
    c = T.KVCache(num_layers=1, num_kv_heads=1, head_dim=64, max_seq_len=64, max_batch_size=2,
                  num_blocks=3)
    a = c.allocate_sequence(64)
    c.allocate_sequence(64)
    k = to_dev(O.normal_f16((40, 1, 64), 1))
    with pytest.raises(T.Exhausted):
        c.append_kv(a, 0, k.data_ptr(), k.data_ptr(), 40)
    assert c.get_seq_len(a) == 0 and len(c.block_table(a)) == 1
    c.sync_check()


def test_all_layer_append_rejects_duplicates_and_overflow():
    c = T.KVCache(num_layers=2, num_kv_heads=1, head_dim=64, max_seq_len=4, max_batch_size=2)
    a = c.allocate_sequence(1)
    k = to_dev(O.normal_f16((2, 2, 1, 64), 1))
    with pytest.raises(T.InvalidArgument):
        c.append_kv_all_layers([a, a], k.data_ptr(), k.data_ptr())
    c.append_kv_all_layers([a], k.data_ptr(), k.data_ptr())
    c.advance_seq_len(a, 1)
    with pytest.raises(T.Overflow):
        c.append_kv_all_layers([a], k.data_ptr(), k.data_ptr())
    c.sync_check()


def _qkv_weights(hidden, ncols, group, seed):
    """Seeded int8 weights [hidden][ncols] in [-127, 127] and fp16 scales
    [hidden/group][ncols] in [0.002, 0.02] (the reference's QuantizedWeight
    layout)."""
    rng = np.random.default_rng(seed)
    w = rng.integers(-127, 128, (hidden, ncols), dtype=np.int64).astype(np.int8)
    s = np.float16(rng.uniform(0.002, 0.02, (hidden // group, ncols))).view(np.uint16)
    return w, s


def _close_f16_rows(got, exp, what):
    """fp16 outputs of fp32 sums formed in another order: within two fp16
    units of the row's largest magnitude (a flip of the last rounding, and
    RoPE mixing two such values)."""
    got = O.f16_to_f32(got).astype(np.float64).reshape(exp.shape[0], -1)
    exp = O.f16_to_f32(exp).astype(np.float64).reshape(exp.shape[0], -1)
    tol = 2.0 ** (np.floor(np.log2(np.abs(exp).max(axis=1, keepdims=True) + 1e-30)) - 9)
    bad = np.abs(got - exp) > tol
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {bad.size} outside 2 fp16 units; "
                           f"max err {np.abs(got - exp).max():.3e}")


@pytest.mark.parametrize("D,G,bs,rope,layout,B,hidden,group", [
    (128, 4, 16, True, T.TL_LAYOUT_TOKEN_MAJOR, 5, 512, 32),
    (64, 2, 32, False, T.TL_LAYOUT_HEAD_MAJOR, 17, 256, 16),
    (128, 1, 16, True, T.TL_LAYOUT_HEAD_MAJOR, 33, 1024, 128),
    (64, 8, 16, True, T.TL_LAYOUT_TOKEN_MAJOR, 64, 384, 64),
    (128, 4, 16, False, T.TL_LAYOUT_TOKEN_MAJOR, 70, 256, 32),
    (128, 4, 16, True, T.TL_LAYOUT_TOKEN_MAJOR, 33, 512, 16),
    (128, 2, 16, True, T.TL_LAYOUT_TOKEN_MAJOR, 40, 4096, 32),
    (128, 2, 16, True, T.TL_LAYOUT_HEAD_MAJOR, 50, 4096, 128),
    (128, 4, 32, False, T.TL_LAYOUT_TOKEN_MAJOR, 20, 4096, 64),
])
def test_project_qkv_append(D, G, bs, rope, layout, B, hidden, group):
    """Fused W8A16 Q/K/V projection of one decode token per sequence
    (replacing the decode step's three kernels::w8a16_matmul and appendKV):
    Q and the K/V rows written at each sequence's length match the oracle's
    restatement of the reference matmul rounded to fp16 (then rotated at
    that position when the cache rotates on append); every earlier row of
    the pool is untouched. B = 70 runs as two launches. Group 16 runs the
    mma.sync kernel, the other groups the tcgen05 kernel, except where no
    split of K keeps the group accumulators within TMEM (group 32 with 40
    rows of hidden 4096), which falls back to the mma.sync kernel; hidden
    4096 with groups 64 and 128 runs the tcgen05 kernel at 32 and 64 rows."""
    import torch
    Hkv = 2
    Hq = Hkv * G
    L = 3
    r = Run.create(L=L, Hq=Hq, Hkv=Hkv, D=D, bs=bs, max_seq_len=160, max_batch=B, rope=rope,
                   layout=layout, permute_seed=5)
    lens = [(7 * i + 3) % 97 for i in range(B)]
    sids = [r.allocate(160) for _ in range(B)]
    for i, (sid, P) in enumerate(zip(sids, lens)):
        if P:
            r.prefill(sid, P, seed=300 + i)
    x = O.normal_f16((B, hidden), 77 + B)
    wq, sq = _qkv_weights(hidden, Hq * D, group, 1)
    wk, sk = _qkv_weights(hidden, Hkv * D, group, 2)
    wv, sv = _qkv_weights(hidden, Hkv * D, group, 3)
    dev = [to_dev(a) if a.dtype == np.uint16 else torch.from_numpy(a.copy()).cuda() for a in
           (x, wq, sq, wk, sk, wv, sv)]
    qd = torch.full((B, Hq * D), 0x7e00, dtype=torch.int16, device="cuda")
    layer = 1
    r.cache.project_qkv_append(layer, dev[0].data_ptr(), hidden, dev[1].data_ptr(), dev[2].data_ptr(),
                               dev[3].data_ptr(), dev[4].data_ptr(), dev[5].data_ptr(), dev[6].data_ptr(),
                               group, sids, qd.data_ptr())
    r.cache.sync_check()
    eq = O.f32_to_f16(O.w8a16_matmul(x, wq, sq, group)).reshape(B, Hq, D)
    ek = O.f32_to_f16(O.w8a16_matmul(x, wk, sk, group)).reshape(B, Hkv, D)
    ev = O.f32_to_f16(O.w8a16_matmul(x, wv, sv, group)).reshape(B, Hkv, D)
    if rope:
        eq = np.stack([O.rope_row(eq[i], r.cos, r.sin, lens[i]) for i in range(B)])
        ek = np.stack([O.rope_row(ek[i], r.cos, r.sin, lens[i]) for i in range(B)])
    _close_f16_rows(from_dev(qd).reshape(B, Hq, D).reshape(B * Hq, D), eq.reshape(B * Hq, D), "Q")
    base, n = r.cache.pool()
    pool = d2h(base, n)
    g = O.geom(L, Hkv, D, bs, r.cache.config.num_blocks, layout == T.TL_LAYOUT_HEAD_MAJOR)
    for i, sid in enumerate(sids):
        bt = np.array(r.cache.block_table(sid), np.int32)
        k, v = O.gather(pool, g, bt, layer, lens[i] + 1)
        _close_f16_rows(k[lens[i]], ek[i], f"K row of seq {sid}")
        _close_f16_rows(v[lens[i]], ev[i], f"V row of seq {sid}")
        assert r.cache.get_seq_len(sid) == lens[i]  # the length does not advance
    r.check_pool_bit_exact()  # the prefix rows of every layer are untouched


def _pack_layout(w):
    """numpy restatement of tl_qkv_pack_weight's layout: column tile t,
    64-row block b is 8192 bytes at (t * K / 64 + b) * 8192, row r's 16-byte
    chunk c at r * 128 + (c ^ (r % 8)) * 16."""
    K, n = w.shape
    t = w.reshape(K // 64, 64, n // 128, 8, 16).transpose(2, 0, 1, 3, 4)  # [tile][block][row][chunk][16]
    rows = np.arange(64)[:, None]
    src_chunk = np.arange(8)[None, :] ^ (rows & 7)  # position p holds chunk p ^ (r % 8)
    return np.ascontiguousarray(t[:, :, rows, src_chunk, :]).reshape(-1)


@pytest.mark.parametrize("D,G,bs,rope,layout,B,hidden,group", [
    (128, 4, 16, True, T.TL_LAYOUT_TOKEN_MAJOR, 5, 512, 32),
    (64, 8, 16, True, T.TL_LAYOUT_TOKEN_MAJOR, 64, 384, 64),
    (128, 4, 16, False, T.TL_LAYOUT_TOKEN_MAJOR, 70, 256, 32),
    (128, 2, 16, True, T.TL_LAYOUT_HEAD_MAJOR, 50, 4096, 128),
    (128, 4, 32, False, T.TL_LAYOUT_TOKEN_MAJOR, 20, 4096, 64),
])
def test_project_qkv_append_packed(D, G, bs, rope, layout, B, hidden, group):
    """Weights repacked on the device by tl_qkv_pack_weight equal the numpy
    restatement of the tile-blocked layout byte for byte; the projection
    from them (tl_project_qkv_append_packed) writes Q and every sequence's
    K/V row within two fp16 units of the oracle, as tl_project_qkv_append
    does from the reference layout, and leaves every other pool row
    untouched. (Split-K partial sums meet in L2 in arrival order, so two
    runs of either entry may differ in the last bit; the oracle is the
    check.) B = 70 runs as two launches; hidden 4096 runs 16-way split-K."""
    import torch
    Hkv = 2
    Hq = Hkv * G
    L = 2
    r = Run.create(L=L, Hq=Hq, Hkv=Hkv, D=D, bs=bs, max_seq_len=160, max_batch=B, rope=rope,
                   layout=layout, permute_seed=9)
    lens = [(5 * i + 2) % 89 for i in range(B)]
    sids = [r.allocate(160) for _ in range(B)]
    for i, (sid, P) in enumerate(zip(sids, lens)):
        if P:
            r.prefill(sid, P, seed=500 + i)
    x = O.normal_f16((B, hidden), 91 + B)
    ws = [_qkv_weights(hidden, nc, group, 11 + j) for j, nc in enumerate((Hq * D, Hkv * D, Hkv * D))]
    xd = to_dev(x)
    wd = [torch.from_numpy(w.copy()).cuda() for w, _ in ws]
    sd = [to_dev(sc) for _, sc in ws]
    packed = [torch.empty_like(w) for w in wd]
    for w, p in zip(wd, packed):
        T.pack_qkv_weight(w.data_ptr(), hidden, w.shape[1], p.data_ptr())
    torch.cuda.synchronize()
    for (w, _), p in zip(ws, packed):
        assert np.array_equal(p.cpu().numpy().reshape(-1), _pack_layout(w)), "packed layout differs"
    del wd
    layer = 1
    qd = torch.full((B, Hq * D), 0x7e00, dtype=torch.int16, device="cuda")
    r.cache.project_qkv_append_packed(layer, xd.data_ptr(), hidden, packed[0].data_ptr(), sd[0].data_ptr(),
                                      packed[1].data_ptr(), sd[1].data_ptr(), packed[2].data_ptr(),
                                      sd[2].data_ptr(), group, sids, qd.data_ptr())
    r.cache.sync_check()
    eq, ek, ev = (O.f32_to_f16(O.w8a16_matmul(x, w, sc, group)).reshape(B, -1, D) for w, sc in ws)
    if rope:
        eq = np.stack([O.rope_row(eq[i], r.cos, r.sin, lens[i]) for i in range(B)])
        ek = np.stack([O.rope_row(ek[i], r.cos, r.sin, lens[i]) for i in range(B)])
    _close_f16_rows(from_dev(qd).reshape(B * Hq, D), eq.reshape(B * Hq, D), "Q")
    base, n = r.cache.pool()
    pool = d2h(base, n)
    g = O.geom(L, Hkv, D, bs, r.cache.config.num_blocks, layout == T.TL_LAYOUT_HEAD_MAJOR)
    for i, sid in enumerate(sids):
        bt = np.array(r.cache.block_table(sid), np.int32)
        k, v = O.gather(pool, g, bt, layer, lens[i] + 1)
        _close_f16_rows(k[lens[i]], ek[i], f"K row of seq {sid}")
        _close_f16_rows(v[lens[i]], ev[i], f"V row of seq {sid}")
        assert r.cache.get_seq_len(sid) == lens[i]
    r.check_pool_bit_exact()


@pytest.mark.parametrize("packed", [False, True])
def test_project_qkv_append_llama3_shape(packed):
    """The bench's shape (Llama-3-8B: 32 query heads, 8 KV heads, D 128,
    hidden 4096, group 128, 32 sequences, RoPE): K is split six ways into
    chunks of 11 blocks of 64 rows, which start and end inside scale groups;
    Q and every sequence's K/V row within two fp16 units of the oracle,
    from the reference layout and from packed weights."""
    import torch
    B, Hq, Hkv, D, hidden, group = 32, 32, 8, 128, 4096, 128
    r = Run.create(L=2, Hq=Hq, Hkv=Hkv, D=D, bs=16, max_seq_len=96, max_batch=B, rope=True,
                   layout=T.TL_LAYOUT_TOKEN_MAJOR, permute_seed=3)
    lens = [(11 * i + 5) % 80 for i in range(B)]
    sids = [r.allocate(96) for _ in range(B)]
    for i, (sid, P) in enumerate(zip(sids, lens)):
        if P:
            r.prefill(sid, P, seed=700 + i)
    x = O.normal_f16((B, hidden), 123)
    ws = [_qkv_weights(hidden, nc, group, 31 + j) for j, nc in enumerate((Hq * D, Hkv * D, Hkv * D))]
    xd = to_dev(x)
    wd = [torch.from_numpy(w.copy()).cuda() for w, _ in ws]
    sd = [to_dev(sc) for _, sc in ws]
    if packed:
        pk = [torch.empty_like(w) for w in wd]
        for w, p in zip(wd, pk):
            T.pack_qkv_weight(w.data_ptr(), hidden, w.shape[1], p.data_ptr())
        wd = pk
    layer = 0
    qd = torch.full((B, Hq * D), 0x7e00, dtype=torch.int16, device="cuda")
    proj = r.cache.project_qkv_append_packed if packed else r.cache.project_qkv_append
    proj(layer, xd.data_ptr(), hidden, wd[0].data_ptr(), sd[0].data_ptr(), wd[1].data_ptr(), sd[1].data_ptr(),
         wd[2].data_ptr(), sd[2].data_ptr(), group, sids, qd.data_ptr())
    r.cache.sync_check()
    eq, ek, ev = (O.f32_to_f16(O.w8a16_matmul(x, w, sc, group)).reshape(B, -1, D) for w, sc in ws)
    eq = np.stack([O.rope_row(eq[i], r.cos, r.sin, lens[i]) for i in range(B)])
    ek = np.stack([O.rope_row(ek[i], r.cos, r.sin, lens[i]) for i in range(B)])
    _close_f16_rows(from_dev(qd).reshape(B * Hq, D), eq.reshape(B * Hq, D), "Q")
    base, n = r.cache.pool()
    pool = d2h(base, n)
    g = O.geom(2, Hkv, D, 16, r.cache.config.num_blocks, False)
    for i, sid in enumerate(sids):
        bt = np.array(r.cache.block_table(sid), np.int32)
        k, v = O.gather(pool, g, bt, layer, lens[i] + 1)
        _close_f16_rows(k[lens[i]], ek[i], f"K row of seq {sid}")
        _close_f16_rows(v[lens[i]], ev[i], f"V row of seq {sid}")
    r.check_pool_bit_exact()


@pytest.mark.parametrize("D,G,B,hidden,group,rope,packed", [
    (128, 4, 20, 1152, 128, True, False),   # chunks of 3 blocks: scale groups split between CTAs
    (64, 8, 16, 384, 64, True, True),       # six CTAs of one block each
    (128, 2, 32, 640, 128, False, True),    # five CTAs of two blocks
    (128, 4, 1, 4096, 128, True, False),    # one row
])
def test_project_qkv_append_split_shapes(D, G, B, hidden, group, rope, packed):
    """K-splits whose chunks split scale groups between CTAs, one-block
    chunks, an uneven last chunk and a single row: Q and every K/V row
    within two fp16 units of the oracle, and the rest of the pool
    untouched."""
    import torch
    Hkv = 2
    Hq = Hkv * G
    r = Run.create(L=2, Hq=Hq, Hkv=Hkv, D=D, bs=16, max_seq_len=96, max_batch=B, rope=rope,
                   layout=T.TL_LAYOUT_TOKEN_MAJOR, permute_seed=4)
    lens = [(13 * i + 1) % 70 for i in range(B)]
    sids = [r.allocate(96) for _ in range(B)]
    for i, (sid, P) in enumerate(zip(sids, lens)):
        if P:
            r.prefill(sid, P, seed=900 + i)
    x = O.normal_f16((B, hidden), 321 + B)
    ws = [_qkv_weights(hidden, nc, group, 51 + j) for j, nc in enumerate((Hq * D, Hkv * D, Hkv * D))]
    xd = to_dev(x)
    wd = [torch.from_numpy(w.copy()).cuda() for w, _ in ws]
    sd = [to_dev(sc) for _, sc in ws]
    if packed:
        pk = [torch.empty_like(w) for w in wd]
        for w, p in zip(wd, pk):
            T.pack_qkv_weight(w.data_ptr(), hidden, w.shape[1], p.data_ptr())
        wd = pk
    layer = 1
    qd = torch.full((B, Hq * D), 0x7e00, dtype=torch.int16, device="cuda")
    proj = r.cache.project_qkv_append_packed if packed else r.cache.project_qkv_append
    proj(layer, xd.data_ptr(), hidden, wd[0].data_ptr(), sd[0].data_ptr(), wd[1].data_ptr(), sd[1].data_ptr(),
         wd[2].data_ptr(), sd[2].data_ptr(), group, sids, qd.data_ptr())
    r.cache.sync_check()
    eq, ek, ev = (O.f32_to_f16(O.w8a16_matmul(x, w, sc, group)).reshape(B, -1, D) for w, sc in ws)
    if rope:
        eq = np.stack([O.rope_row(eq[i], r.cos, r.sin, lens[i]) for i in range(B)])
        ek = np.stack([O.rope_row(ek[i], r.cos, r.sin, lens[i]) for i in range(B)])
    _close_f16_rows(from_dev(qd).reshape(B * Hq, D), eq.reshape(B * Hq, D), "Q")
    base, n = r.cache.pool()
    pool = d2h(base, n)
    g = O.geom(2, Hkv, D, 16, r.cache.config.num_blocks, False)
    for i, sid in enumerate(sids):
        bt = np.array(r.cache.block_table(sid), np.int32)
        k, v = O.gather(pool, g, bt, layer, lens[i] + 1)
        _close_f16_rows(k[lens[i]], ek[i], f"K row of seq {sid}")
        _close_f16_rows(v[lens[i]], ev[i], f"V row of seq {sid}")
    r.check_pool_bit_exact()


def test_project_qkv_append_packed_refuses_other_shapes():
    """Group 16 (the mma.sync kernel's shape) has no packed form: the
    packed entry refuses it before any launch."""
    import torch
    r = Run.create(L=1, Hq=8, Hkv=2, D=128, bs=16, max_seq_len=64, max_batch=2, rope=False)
    sids = [r.allocate(64) for _ in range(2)]
    buf = torch.zeros(1 << 20, dtype=torch.int8, device="cuda")
    p = buf.data_ptr()
    with pytest.raises(T.Unsupported) as e:
        r.cache.project_qkv_append_packed(0, p, 256, p, p, p, p, p, p, 16, sids, p)
    assert "packed weights need" in str(e.value)
    r.cache.sync_check()
