"""Multi-rank host logic on CPU: two gloo ranks (spawned processes).

Covers the head/batch sharding, the max/sum timing reductions and the
rank-major all-gather layout of the head-sharded decode: each rank computes
its heads' outputs with the CPU oracle, the slices are all-gathered, and the
reassembled [B][Hq][D] must equal the single-process oracle output. A rank
that fails before a collective makes the other rank's collective raise
(bounded by the process-group timeout) instead of hanging.
"""
import datetime
import math
import multiprocessing as mp
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tiny-llm_b200" / "python"))
sys.path.insert(0, str(ROOT / "oracle"))

from tiny_llm_b200 import dist as D  # noqa: E402


def test_head_shard_covers_every_head_once():
    for world in (1, 2, 4, 8):
        kv, q = [], []
        for r in range(world):
            s = D.head_shard(8, 64, world, r)
            kv += list(range(s.kv_first, s.kv_first + s.kv_count))
            q += list(range(s.q_first, s.q_first + s.q_count))
            # the query heads of a slice are exactly those reading its KV heads (q // G)
            assert {h // 8 for h in range(s.q_first, s.q_first + s.q_count)} == \
                set(range(s.kv_first, s.kv_first + s.kv_count))
        assert kv == list(range(8)) and q == list(range(64))
    with pytest.raises(ValueError):
        D.head_shard(8, 64, 3, 0)


def test_batch_shard_balances_kv_bytes():
    rng = np.random.default_rng(0)
    lens = [int(x) for x in rng.integers(512, 8193, size=64)]
    for world in (1, 2, 4, 8):
        parts = D.batch_shard(lens, world)
        assert sorted(i for p in parts for i in p) == list(range(64))
        loads = [sum(lens[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(lens)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, scenario, q_out):
    import torch
    import torch.distributed as dist
    sys.path.insert(0, str(ROOT / "tiny-llm_b200" / "python"))
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle as O
    from tiny_llm_b200 import dist as DD
    try:
        if scenario == "fail" and rank == 1:
            raise RuntimeError("rank 1 fails before joining the collective")
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=8))
        if scenario == "dies":
            if rank == 1:
                q_out.put((rank, "exited"))
                q_out.close()
                q_out.join_thread()  # flush the message before leaving
                import os
                os._exit(0)  # leaves between steps, with no collective in flight
            try:
                DD.reduce_max(1.0)
                q_out.put((rank, "no-error"))
            except Exception as e:
                q_out.put((rank, "error:" + type(e).__name__))
            return
        if scenario == "fail":
            try:
                DD.reduce_max(1.0)
                q_out.put((rank, "no-error"))
            except Exception as e:  # the peer never joined
                q_out.put((rank, "error:" + type(e).__name__))
            return
        mx = DD.reduce_max(float(rank + 1))
        sm = DD.reduce_sum(float(rank + 1))
        B, Hq, Hkv, Dd, S = 2, 8, 2, 64, 37
        sl = DD.head_shard(Hkv, Hq, world, rank)
        scale = 1.0 / math.sqrt(Dd)
        outs = []
        for b in range(B):
            q = O.normal_f16((Hq, Dd), 10 + b)
            k = O.normal_f16((S, Hkv, Dd), 20 + b)
            v = O.normal_f16((S, Hkv, Dd), 30 + b)
            # this rank sees only its KV heads and the query heads reading them
            qs = q[sl.q_first: sl.q_first + sl.q_count]
            ks = k[:, sl.kv_first: sl.kv_first + sl.kv_count]
            vs = v[:, sl.kv_first: sl.kv_first + sl.kv_count]
            outs.append(O.decode_one(qs, ks, vs, scale))
        local = torch.from_numpy(np.stack(outs))            # [B][Hq/N][D]
        gathered = torch.empty((world,) + tuple(local.shape), dtype=local.dtype)
        DD.gather_head_outputs(local, gathered)
        full = DD.rank_major_to_heads(gathered).numpy()      # [B][Hq][D]
        ref = []
        for b in range(B):
            q = O.normal_f16((Hq, Dd), 10 + b)
            k = O.normal_f16((S, Hkv, Dd), 20 + b)
            v = O.normal_f16((S, Hkv, Dd), 30 + b)
            ref.append(O.decode_one(q, k, v, scale))
        ok = bool(np.array_equal(full, np.stack(ref)))
        q_out.put((rank, (mx, sm, ok)))
        dist.destroy_process_group()
    except Exception as e:
        q_out.put((rank, "exception:" + repr(e)))


def _run(world, scenario, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, scenario, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, val = q.get(timeout=timeout)
        results[r] = val
    for p in procs:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return results


def test_two_rank_reductions_and_head_gather_layout():
    res = _run(2, "ok")
    for r in (0, 1):
        mx, sm, ok = res[r]
        assert mx == 2.0 and sm == 3.0
        assert ok, f"rank {r}: gathered head slices differ from the full oracle output"


def test_rank_that_never_joins_makes_the_others_raise_not_hang():
    res = _run(2, "fail")
    assert res[1].startswith("exception:") and "fails before" in res[1]
    # rank 0 learns of it on the host: the rendezvous times out with an error
    assert res[0].startswith("exception:") or res[0].startswith("error:"), res[0]


def test_rank_that_exits_between_steps_makes_the_next_collective_raise():
    res = _run(2, "dies")
    assert res[1] == "exited"
    assert res[0].startswith("error:"), res[0]


def test_bench_strong_scaling_splits_the_config_batch():
    """bench.py --gpus N (strong scaling, the default): the ranks' sequences
    together are the config's batch, each exactly once, balanced by KV bytes
    to within one sequence; --scaling weak gives every rank a whole batch."""
    import argparse
    import importlib
    import sys as _sys

    _sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    bench = importlib.import_module("bench")
    for name in ("c2", "c3", "c4", "c5s"):
        cfg = bench.CONFIGS[name]
        full = bench.seq_lens(cfg, 0, 0)
        for world in (1, 2, 4, 8):
            args = argparse.Namespace(seed=0, scaling="strong")
            parts = [bench.rank_lens(cfg, args, world, r) for r in range(world)]
            assert all(gb == len(full) for _, gb in parts)
            assert sorted(x for lens, _ in parts for x in lens) == sorted(full)
            loads = [sum(lens) for lens, _ in parts]
            assert max(loads) - min(loads) <= max(full), (name, world, loads)
        weak = [bench.rank_lens(cfg, argparse.Namespace(seed=0, scaling="weak"), 4, r) for r in range(4)]
        assert all(len(lens) == len(full) and gb == 4 * len(full) for lens, gb in weak)
