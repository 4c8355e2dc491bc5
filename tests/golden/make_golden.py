"""Generates the golden fixtures of tests/golden/ by running the REFERENCE's
own CUDA code (oracle/_ref/libtllm_ref.so, built from the reference sources
by oracle/Makefile.ref) on seeded inputs. Needs a GPU; run on the GPU box:

    python tests/golden/make_golden.py [out_dir]

which writes the *.npz files to out_dir (default: tests/golden/ itself). Inputs are regenerated from
their seeds by the oracle's generator (oracle.normal_f16); each fixture stores
the seeds, shapes, a SHA-256 of the generated inputs (to catch generator
drift) and the reference's outputs.

decode_*: kernels::attention_decode (kernels/attention.cu:114-128) on
  [B][Hq][S][D] K/V. GQA cases give the MHA-only kernel K/V expanded per
  query head, so its output is the GQA attention of the un-expanded K/V.
append_*: KVCacheManager::appendKV / advanceSeqLen (src/kv_cache.cpp:168-259)
  followed by a read-back of getCache() for every layer of the sequence.
"""
from __future__ import annotations

import hashlib
import math
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1] / "oracle"))
sys.path.insert(0, str(HERE))

import oracle as O  # noqa: E402
import ref_lib  # noqa: E402

DECODE_CASES = [
    # name, B, Hq, Hkv, S, D, seed
    ("decode_mha_s17_d64", 2, 4, 4, 17, 64, 11),
    ("decode_mha_s300_d128", 1, 8, 8, 300, 128, 12),
    ("decode_gqa4_s1000_d128", 2, 8, 2, 1000, 128, 13),
    ("decode_gqa8_s129_d128", 1, 16, 2, 129, 128, 14),
    ("decode_mha_s1_d64", 3, 2, 2, 1, 64, 15),
]


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def decode_inputs(B, Hq, Hkv, S, D, seed):
    q = O.normal_f16((B, Hq, D), seed * 100 + 1)
    k = O.normal_f16((B, S, Hkv, D), seed * 100 + 2)
    v = O.normal_f16((B, S, Hkv, D), seed * 100 + 3)
    return q, k, v


def expand_for_reference(x, Hq):
    """[B][S][Hkv][D] -> the reference kernel's [B][Hq][S][D], head hq reading kv head hq/G."""
    B, S, Hkv, D = x.shape
    G = Hq // Hkv
    return np.ascontiguousarray(np.repeat(x.transpose(0, 2, 1, 3), G, axis=1))


def main(out: Path):
    import torch

    out.mkdir(parents=True, exist_ok=True)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).cuda()
    for name, B, Hq, Hkv, S, D, seed in DECODE_CASES:
        q, k, v = decode_inputs(B, Hq, Hkv, S, D, seed)
        qd, kd, vd = dev(q), dev(expand_for_reference(k, Hq)), dev(expand_for_reference(v, Hq))
        od = torch.zeros((B, Hq, D), dtype=torch.int16, device="cuda")
        scale = 1.0 / math.sqrt(D)
        ref_lib.attention_decode(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), od.data_ptr(),
                                 scale, B, Hq, S, D)
        torch.cuda.synchronize()
        np.savez(out / f"{name}.npz", shape=np.array([B, Hq, Hkv, S, D, seed]), scale=np.float32(scale),
                 input_sha256=np.array(sha(q, k, v)), out=od.cpu().numpy().view(np.uint16))
        print("wrote", name)

    # append: 2 layers, 4 KV heads, D=32; append 3 tokens, advance 3, append 2
    # more (positions 3,4), advance 2, then read back 5 tokens per layer.
    L, H, D = 2, 4, 32
    rc = ref_lib.RefCache(L, H, D, 64, 2)
    sid = rc.allocate(32)
    ks = O.normal_f16((L, 5, H, D), 900)
    vs = O.normal_f16((L, 5, H, D), 901)
    # keep every device buffer alive until the copies have run: appendKV's
    # memcpys are asynchronous and a freed buffer would be reused at once
    kd1 = [dev(ks[l, :3]) for l in range(L)]
    vd1 = [dev(vs[l, :3]) for l in range(L)]
    for l in range(L):
        rc.append(sid, l, kd1[l].data_ptr(), vd1[l].data_ptr(), 3)
    rc.advance(sid, 3)
    kd2 = [dev(ks[l, 3:]) for l in range(L)]
    vd2 = [dev(vs[l, 3:]) for l in range(L)]
    for l in range(L):
        rc.append(sid, l, kd2[l].data_ptr(), vd2[l].data_ptr(), 2)
    rc.advance(sid, 2)
    torch.cuda.synchronize()
    got_k = np.zeros((L, 5, H, D), np.uint16)
    got_v = np.zeros((L, 5, H, D), np.uint16)
    for l in range(L):
        kp, vp = rc.get_cache(sid, l)
        got_k[l] = ref_lib.d2h(kp, 5 * H * D).reshape(5, H, D)
        got_v[l] = ref_lib.d2h(vp, 5 * H * D).reshape(5, H, D)
    rc.close()
    np.savez(out / "append_l2_h4_d32.npz", shape=np.array([L, H, D, 5]), seeds=np.array([900, 901]),
             input_sha256=np.array(sha(ks, vs)), k=got_k, v=got_v)
    print("wrote append_l2_h4_d32")


if __name__ == "__main__":
    # output directory: the first argument, else the fixtures' own directory
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).resolve().parent)
