"""Head-sharded decode on 2, 4 and 8 GPUs (one process per GPU, NCCL): each
rank appends and decodes only its KV heads (8 KV heads, 32 query heads: 4, 2
or 1 KV head per rank) through the C-ABI, the per-layer outputs are gathered
— by NCCL all-gather, and by the NVLink publish-then-pull fused into the
decode call, which at 4 and 8 ranks pulls several remote slices — and every
rank's reassembled [B][Hq][D] must match the fp64 oracle of the full model
within the attention tolerance. Each world is skipped with fewer GPUs. NVLS
is off, as for every multi-GPU test here. Each rank's worst max-abs and
max-rel error is printed (run with -s to see them)."""
import math
import multiprocessing as mp
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

import conftest

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, q_out):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    sys.path.insert(0, str(ROOT / "tiny-llm_b200" / "python"))
    sys.path.insert(0, str(ROOT / "oracle"))
    sys.path.insert(0, str(ROOT / "tests"))
    try:
        import datetime
        import torch
        import torch.distributed as dist
        import oracle as O
        import tiny_llm_b200 as T
        from tiny_llm_b200 import dist as TD
        from gpu_helpers import check_close, from_dev, to_dev
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        L, Hq, Hkv, D, bs = 2, 32, 8, 128, 32
        lens = [700, 33, 1500]
        sl = TD.head_shard(Hkv, Hq, world, rank)
        cache = T.KVCache(num_layers=L, num_kv_heads=sl.kv_count, head_dim=D, max_seq_len=2048,
                          max_batch_size=len(lens), block_size=bs, num_q_heads=sl.q_count,
                          rope_on_append=True, device=rank)
        cos, sin = O.rope_table(2048, D, 10000.0)
        full_k, full_v = {}, {}
        sids = []
        keep = []
        for i, S in enumerate(lens):
            sid = cache.allocate_sequence(2048)
            sids.append(sid)
            for l in range(L):
                k = O.normal_f16((S, Hkv, D), 1000 * i + 2 * l)
                v = O.normal_f16((S, Hkv, D), 1000 * i + 2 * l + 1)
                full_k[(i, l)] = np.stack([O.rope_row(k[t], cos, sin, t) for t in range(S)])
                full_v[(i, l)] = v
                ks = to_dev(np.ascontiguousarray(k[:, sl.kv_first: sl.kv_first + sl.kv_count]))
                vs = to_dev(np.ascontiguousarray(v[:, sl.kv_first: sl.kv_first + sl.kv_count]))
                keep += [ks, vs]
                cache.append_kv(sid, l, ks.data_ptr(), vs.data_ptr(), S)
            cache.advance_seq_len(sid, S)
        scale = 1.0 / math.sqrt(D)
        worst = [0.0, 0.0]

        def note(ma_mr):
            worst[0], worst[1] = max(worst[0], ma_mr[0]), max(worst[1], ma_mr[1])

        for l in range(L):
            q = O.normal_f16((len(lens), Hq, D), 77 + l)
            qs = to_dev(np.ascontiguousarray(q[:, sl.q_first: sl.q_first + sl.q_count]))
            o = torch.empty((len(lens), sl.q_count, D), dtype=torch.float16, device="cuda")
            cache.decode_attention(l, qs.data_ptr(), o.data_ptr(), sids, scale)
            gathered = torch.empty((world, len(lens), sl.q_count, D), dtype=torch.float16, device="cuda")
            TD.gather_head_outputs(o, gathered)
            full = TD.rank_major_to_heads(gathered)
            cache.sync_check()
            got = O.f16_to_f32(from_dev(full))
            for i in range(len(lens)):
                ref = O.decode_one(q[i], full_k[(i, l)], full_v[(i, l)], scale)
                note(check_close(got[i], ref, f"rank {rank} layer {l} seq {i}"))
        # the same layers through the NVLink peer-store gather
        from gpu_helpers import d2h
        slice_bytes = len(lens) * sl.q_count * D * 2
        TD.connect_peer_gather(cache, L * world * slice_bytes)
        gptr, _ = cache.peer_buffer()
        dist.barrier()  # both ranks reach the GPU-side waits together
        qkeep = []
        for l in range(L):
            q = O.normal_f16((len(lens), Hq, D), 77 + l)
            qs = to_dev(np.ascontiguousarray(q[:, sl.q_first: sl.q_first + sl.q_count]))
            qkeep.append(qs)
            cache.decode_attention_peer(l, qs.data_ptr(), sids, l * world * slice_bytes, l + 1, scale)
        cache.sync_check()
        for l in range(L):
            q = O.normal_f16((len(lens), Hq, D), 77 + l)
            g = d2h(gptr + l * world * slice_bytes, world * slice_bytes // 2)
            full = g.reshape(world, len(lens), sl.q_count, D).transpose(1, 0, 2, 3).reshape(len(lens), Hq, D)
            got = O.f16_to_f32(np.ascontiguousarray(full))
            for i in range(len(lens)):
                ref = O.decode_one(q[i], full_k[(i, l)], full_v[(i, l)], scale)
                note(check_close(got[i], ref, f"peer gather: rank {rank} layer {l} seq {i}"))
        dist.barrier()
        cache.close()
        dist.destroy_process_group()
        q_out.put((rank, f"ok max_abs={worst[0]:.3e} max_rel={worst[1]:.3e}"))
    except Exception as e:
        q_out.put((rank, "fail: " + repr(e)))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_head_sharded_decode(world):
    if not conftest.cuda_available():
        pytest.skip("no CUDA device")
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    for r in sorted(res):
        print(f"head shard world {world} rank {r}: {res[r]}")
    assert all(res.get(r, "").startswith("ok") for r in range(world)), res
