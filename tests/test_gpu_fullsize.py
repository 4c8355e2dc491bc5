"""Parity at the BASELINE configs' full sizes (c2, c3, c4 on one GPU, and
config 5's steady-state batch of 225 short sequences).

The whole batch is prefilled through the per-layer append (RoPE on K), one
fused all-layer append step is applied, and decode runs on the sampled layers
for every sequence. Checked on a sample of (sequence, layer) units, because
the fp64 oracle cannot redo 30-90 GB of attention in a test:
  * the pool gathered through the block table equals the regenerated inputs
    (K rotated by the oracle's RoPE) bit for bit;
  * decode output equals the fp64 oracle on the gathered K/V within
    |got - ref| <= 2e-3 + 1e-3|ref|.
"""
import math

import numpy as np
import pytest

import conftest
import oracle as O
import tiny_llm_b200 as T
from gpu_helpers import check_close, d2h, from_dev

pytestmark = pytest.mark.gpu

CASES = {
    # name: L, Hq, Hkv, D, bs, lens, permute
    "c2": (32, 32, 32, 128, 16, [2048] * 32, False),
    "c3": (32, 32, 8, 128, 16, "ragged", True),
    "c4": (80, 64, 8, 128, 32, [32768] * 8, False),
    # config 5's steady-state decode batch: 225 sequences, log-uniform
    # prompts in [32, 4096] plus half a geometric(256) generation, permuted
    "c5s": (32, 32, 8, 128, 16, "loguniform", True),
}


def _loguniform_lens(seed=0, n=225, lo=32, hi=4096):
    rng = np.random.default_rng(seed)
    return [int(round(math.exp(x))) + int(rng.geometric(1 / 256)) // 2
            for x in rng.uniform(math.log(lo), math.log(hi), size=n)]


def _kv_chunk(torch, sid, layer, P, Hkv, D):
    g = torch.Generator(device="cuda")
    g.manual_seed(1_000_003 * (sid + 1) + layer)
    return torch.randn((2, P, Hkv, D), dtype=torch.float16, device="cuda", generator=g)


@pytest.mark.parametrize("name", sorted(CASES))
def test_full_size_config(name):
    if not conftest.cuda_available():
        pytest.skip("no CUDA device")
    import torch

    L, Hq, Hkv, D, bs, lens, permute = CASES[name]
    if lens == "ragged":
        lens = [int(x) for x in np.random.default_rng(0).integers(512, 8193, size=64)]
    elif lens == "loguniform":
        lens = _loguniform_lens()
    B = len(lens)
    max_len = max(lens) + 4
    nblocks = sum(-(-(l + 4) // bs) for l in lens)
    cache = T.KVCache(num_layers=L, num_kv_heads=Hkv, head_dim=D, max_seq_len=max_len,
                      max_batch_size=B, block_size=bs, num_blocks=nblocks, num_q_heads=Hq,
                      rope_on_append=True, rope_theta=10000.0)
    if permute:
        cache.permute_free_blocks(7)
    sids = [cache.allocate_sequence(max_len) for _ in range(B)]
    for sid, P in zip(sids, lens):
        for l in range(L):
            kv = _kv_chunk(torch, sid, l, P, Hkv, D)
            cache.append_kv(sid, l, kv[0].data_ptr(), kv[1].data_ptr(), P)
        cache.advance_seq_len(sid, P)
    step = torch.randn((2, L, B, Hkv, D), dtype=torch.float16, device="cuda",
                       generator=torch.Generator(device="cuda").manual_seed(5))
    cache.append_kv_all_layers(sids, step[0].data_ptr(), step[1].data_ptr())
    cache.sync_check()

    rng = np.random.default_rng(1)
    nsample = 8 if B > 100 else 3  # many short sequences: sample more of them
    sample = sorted({(int(rng.integers(B)), int(rng.integers(L))) for _ in range(nsample)})
    cos, sin = O.rope_table(max_len, D, 10000.0)
    base, _ = cache.pool()
    cfg = cache.config
    block_elems = bs * Hkv * D
    scale = 1.0 / math.sqrt(D)
    step_np = step.cpu().numpy().view(np.uint16)
    for layer in sorted({l for _, l in sample}):
        q = torch.randn((B, Hq, D), dtype=torch.float16, device="cuda",
                        generator=torch.Generator(device="cuda").manual_seed(100 + layer))
        o = torch.full((B, Hq, D), float("nan"), dtype=torch.float16, device="cuda")
        cache.decode_attention(layer, q.data_ptr(), o.data_ptr(), sids, scale)
        cache.sync_check()
        got = o.float().cpu().numpy()
        qn = q.cpu().numpy().view(np.uint16)
        for b in sorted({b for b, l in sample if l == layer}):
            sid, P = sids[b], lens[b]
            S = P + 1
            bt = np.array(cache.block_table(sid), np.int32)
            # gather the unit's blocks from the device pool (only those blocks)
            kblk = np.stack([d2h(base + 2 * (((layer * 2 + 0) * cfg.num_blocks + int(x)) * block_elems), block_elems) for x in bt])
            vblk = np.stack([d2h(base + 2 * (((layer * 2 + 1) * cfg.num_blocks + int(x)) * block_elems), block_elems) for x in bt])
            k = kblk.reshape(-1, Hkv, D)[:S]
            v = vblk.reshape(-1, Hkv, D)[:S]
            src = _kv_chunk(torch, sid, layer, P, Hkv, D).cpu().numpy().view(np.uint16)
            src_k = np.concatenate([src[0], step_np[0, layer, b][None]])
            src_v = np.concatenate([src[1], step_np[1, layer, b][None]])
            rk = np.stack([O.rope_row(src_k[t], cos, sin, t) for t in range(S)])
            assert np.array_equal(k, rk), f"{name}: K gather mismatch seq {b} layer {layer}"
            assert np.array_equal(v, src_v), f"{name}: V gather mismatch seq {b} layer {layer}"
            ref = O.decode_one(qn[b], k, v, scale)
            check_close(got[b], ref, f"{name} seq {b} layer {layer} S={S}")
    cache.close()
