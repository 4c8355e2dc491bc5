#!/usr/bin/env python
"""Decode attention + KV append benchmark on B200 (one JSON line on rank 0).

A step = for every sequence of the batch, the fused all-layer KV append of
one token (RoPE on K), then decode attention for every layer over the paged
cache (each sequence attends len+1 tokens), then advanceSeqLen — the
per-token work TransformerLayer::attention does in the reference
(src/transformer.cpp:222-237), for the whole batch. Q/K/V inputs are
pre-generated device buffers (cycled); nothing else is skipped.

Workload (default): Llama-2-7B-shaped MHA, 32 layers,
32 query = 32 KV heads, head_dim 128, fp16, 32 sequences at context 2048,
block 16, RoPE theta 10000 on K at append. KV bytes read per step ~34.4 GB
(far larger than the 126 MB L2, so no flush is needed between steps).

  value     aggregate KV-read GB/s over all ranks (sum of KV bytes / max time)
  e2e       same metric through the C-ABI with per-step pinned-host H2D of
            the step's Q/K/V and D2H of its outputs inside the timed region
  roofline  decode kernel: algorithmic bytes per launch / CUDA-event time,
            from a pass after the timed steps with events around each layer
  cpu_baseline  the CPU oracle (fp32, OpenMP) on a bounded sample

--impl reference runs the reference's own path instead (oracle/_ref:
KVCacheManager::appendKV + kernels::attention_decode, rebuilt for sm_100a).

Multi-GPU (torchrun): by default the config's own batch of sequences is
split over the ranks, balanced by KV bytes (dist.batch_shard: independent
sequences, no data-path collective), so the total work is fixed and the
scaling is strong; --scaling weak gives every rank the whole batch instead.
--shard head splits the KV heads of every sequence over the ranks and
gathers each layer's outputs. Time is the max over ranks; the line also
lists every rank's time.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "tiny-llm_b200" / "python"))
sys.path.insert(0, str(ROOT / "oracle"))

CONFIGS = {
    "c1": dict(workload="c1 tiny GQA plumbing", L=2, Hq=8, Hkv=2, D=64, bs=16,
               lens=[17, 64, 100, 128], rope=False),
    "c2": dict(workload="c2 Llama-2-7B MHA decode, 32 seqs @ ctx 2048", L=32, Hq=32, Hkv=32,
               D=128, bs=16, lens=[2048] * 32, rope=True),
    # Profiling case: every decode launch is identical to c2's (32 seqs x 32
    # heads x 2049 tokens, 1.07 GB of KV), with 2 layers so ~2 GB sits on the GPU.
    "c2l2": dict(workload="c2 per-launch shape, 2 layers (ncu case)", L=2, Hq=32, Hkv=32,
                 D=128, bs=16, lens=[2048] * 32, rope=True),
    "c3": dict(workload="c3 Llama-3-8B GQA ragged, 64 seqs ctx U[512,8192], permuted blocks",
               L=32, Hq=32, Hkv=8, D=128, bs=16, lens="ragged", B=64, lo=512, hi=8192,
               rope=True, permute=True),
    "c4": dict(workload="c4 70B long-context GQA, 8 seqs @ ctx 32768 (1 GPU batch shard)",
               L=80, Hq=64, Hkv=8, D=128, bs=32, lens=[32768] * 8, rope=True),
    # one rank's share of c2 with the batch split over 8 GPUs (4 sequences):
    # the per-rank work of that strong-scaling point, on one GPU
    "c2r8": dict(workload="c2 per-rank share at 8 GPUs (4 seqs @ ctx 2048)", L=32, Hq=32, Hkv=32,
                 D=128, bs=16, lens=[2048] * 4, rope=True),
    "c2r2": dict(workload="c2 per-rank share at 2 GPUs (16 seqs @ ctx 2048)", L=32, Hq=32, Hkv=32,
                 D=128, bs=16, lens=[2048] * 16, rope=True),
    "c3r2": dict(workload="c3-shaped per-rank share at 2 GPUs (32 ragged seqs ctx U[512,8192])",
                 L=32, Hq=32, Hkv=8, D=128, bs=16, lens="ragged", B=32, lo=512, hi=8192,
                 rope=True, permute=True),
    "c2r4": dict(workload="c2 per-rank share at 4 GPUs (8 seqs @ ctx 2048)", L=32, Hq=32, Hkv=32,
                 D=128, bs=16, lens=[2048] * 8, rope=True),
    # one rank's slice of c4 head-sharded over 8 GPUs (1 KV head, its 8 query
    # heads, all 8 sequences): the local work of that mode, on one GPU
    "c4r8": dict(workload="c4 per-rank slice of the 8-way head shard (1 KV head, 8 q heads)",
                 L=80, Hq=8, Hkv=1, D=128, bs=32, lens=[32768] * 8, rope=True),
    # c5's steady-state decode batch as a static batch (diagnostic for c5):
    # 225 sequences, lengths log-uniform in [32, 4096] + a geometric(256) tail
    "c5s": dict(workload="c5 steady-state batch, static: 225 seqs, log-U[32,4096] prompts",
                L=32, Hq=32, Hkv=8, D=128, bs=16, lens="loguniform", B=225, lo=32, hi=4096,
                rope=True, permute=True),
    # Paged prefill (the prompt side of the engine): 8 fresh 4096-token
    # prompts, Llama-3-8B GQA shape; 4 layers (every layer is the same work).
    "pf": dict(workload="prefill: 8 prompts x 4096 tokens, Llama-3-8B GQA, 4 layers",
               L=4, Hq=32, Hkv=8, D=128, bs=16, lens=[4096] * 8, rope=True),
    # The decode step's Q/K/V projections (W8A16, the reference's default
    # group of 128) fused with the append: Llama-3-8B shapes, 32 sequences,
    # every layer with its own weights (26 MB each, 839 MB in all).
    "qkv": dict(workload="decode Q/K/V projection W8A16 (group 128) + append, Llama-3-8B, 32 seqs x 32 layers",
                L=32, Hq=32, Hkv=8, D=128, bs=16, hidden=4096, group=128, lens=[512] * 32, rope=True),
    # Next-token sampling on the device: a decode step's logits for 32
    # sequences over the Llama-3 vocabulary, top-p 0.9 at temperature 0.8.
    "smp": dict(workload="next-token sampling: 32 rows x 128256 fp16 logits, top-p 0.9, T 0.8",
                L=1, Hq=32, Hkv=8, D=128, bs=16, lens=[1] * 32, rope=False, vocab=128256),
    "c5": dict(workload="c5 8B GQA continuous-batching churn: Poisson(4) arrivals, prompts "
                        "log-U[32,4096], geometric(256) generations, <=256 active, pool ~80% occupied",
               L=32, Hq=32, Hkv=8, D=128, bs=16, lens="churn", rope=True, permute=True),
}


def launch_traffic(config):
    """dram bytes read + written by one launch of the config's dominant
    kernel, from the ncu capture recorded in profiles/dram_traffic.json."""
    tp = ROOT / "profiles" / "dram_traffic.json"
    if not tp.exists():
        return None
    return json.loads(tp.read_text()).get(config, {}).get("launch")


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def seq_lens(cfg, seed, rank):
    if cfg["lens"] == "loguniform":
        import numpy as np
        rng = np.random.default_rng(seed + 1000 * rank)
        lo, hi = math.log(cfg["lo"]), math.log(cfg["hi"])
        return [int(round(math.exp(x))) + int(rng.geometric(1 / 256)) // 2
                for x in rng.uniform(lo, hi, size=cfg["B"])]
    if cfg["lens"] == "ragged":
        import numpy as np
        rng = np.random.default_rng(seed + 1000 * rank)
        return [int(x) for x in rng.integers(cfg["lo"], cfg["hi"] + 1, size=cfg["B"])]
    return list(cfg["lens"])


class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons during timing."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,"
              "clocks.mem,temperature.memory")

    def __init__(self, device_index: int):
        self.proc = None
        self.path = None
        try:
            self.path = f"/tmp/tllm_clocks_{os.getpid()}.csv"
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={device_index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        rows = []
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        num = lambda v: float(v) if v.replace(".", "").isdigit() else None
        mem = [num(r[9]) for r in rows if len(r) > 9 and num(r[9]) is not None]
        hbm_t = [num(r[10]) for r in rows if len(r) > 10 and num(r[10]) is not None]
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons, "samples": len(rows),
                "mem_mhz": statistics.median(mem) if mem else None,
                "hbm_temp_c": max(hbm_t) if hbm_t else None}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier_max(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier_sum(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def gather_values(value: float, world: int) -> list[float]:
    """Every rank's value of a host scalar, in rank order."""
    if world == 1:
        return [value]
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(x.item()) for x in out]


def rank_lens(cfg, args, world, rank):
    """(sequence lengths this rank decodes, global batch). Strong scaling
    (the default): the config's own batch split over the ranks, balanced by
    KV bytes (dist.batch_shard); weak: every rank runs a whole batch."""
    if world == 1 or args.scaling == "weak":
        lens = seq_lens(cfg, args.seed, rank)
        return lens, len(lens) * world
    from tiny_llm_b200 import dist as TD
    all_lens = seq_lens(cfg, args.seed, 0)
    mine = TD.batch_shard(all_lens, world)[rank]
    if not mine:
        raise SystemExit(f"{len(all_lens)} sequences do not give every one of {world} ranks a sequence")
    return [all_lens[i] for i in mine], len(all_lens)


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def kv_bytes(lens_attended, cfg):
    return sum(lens_attended) * cfg["L"] * 2 * cfg["Hkv"] * cfg["D"] * 2


# --------------------------------------------------------------- our path --

def run_ours(cfg, args, world, rank, local):
    import torch
    import tiny_llm_b200 as T

    from tiny_llm_b200 import dist as TD

    L, Hq, Hkv, D, bs = cfg["L"], cfg["Hq"], cfg["Hkv"], cfg["D"], cfg["bs"]
    head = args.shard == "head"
    if head:
        # every rank holds all sequences but only its slice of the KV heads
        # (and the query heads reading them); outputs are all-gathered
        sl = TD.head_shard(Hkv, Hq, world, rank)
        Hkv, Hq = sl.kv_count, sl.q_count
        lens = seq_lens(cfg, args.seed, 0)
        global_b = len(lens)
    else:
        lens, global_b = rank_lens(cfg, args, world, rank)
    kcfg = dict(cfg, Hkv=Hkv, Hq=Hq)
    B = len(lens)
    steps = args.warmup + args.steps
    e2e_steps = args.warmup + args.steps
    extra = steps + e2e_steps + args.steps + 2  # timed, e2e and roofline passes
    max_len = max(lens) + extra
    layout = T.TL_LAYOUT_HEAD_MAJOR if args.layout == "head" else T.TL_LAYOUT_TOKEN_MAJOR
    nblocks = sum(-(-(l + extra) // bs) for l in lens)
    cache = T.KVCache(num_layers=L, num_kv_heads=Hkv, head_dim=D, max_seq_len=max_len,
                      max_batch_size=B, block_size=bs, num_blocks=nblocks, num_q_heads=Hq,
                      rope_on_append=cfg["rope"], rope_theta=10000.0, layout=layout,
                      device=local)
    if cfg.get("permute"):
        cache.permute_free_blocks(args.seed + rank)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(args.seed * 7919 + rank)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    sids = [cache.allocate_sequence(max_len) for _ in range(B)]
    # Prefill every layer of every sequence through the per-layer append.
    for sid, P in zip(sids, lens):
        for l in range(L):
            kv = torch.randn((2, P, Hkv, D), dtype=torch.float16, device="cuda", generator=gen)
            cache.append_kv(sid, l, kv[0].data_ptr(), kv[1].data_ptr(), P, sp)
        cache.advance_seq_len(sid, P)
    cache.sync_check(sp)

    nbuf = 2
    knew = [torch.randn((L, B, Hkv, D), dtype=torch.float16, device="cuda", generator=gen) for _ in range(nbuf)]
    vnew = [torch.randn((L, B, Hkv, D), dtype=torch.float16, device="cuda", generator=gen) for _ in range(nbuf)]
    q = [torch.randn((L, B, Hq, D), dtype=torch.float16, device="cuda", generator=gen) for _ in range(nbuf)]
    out = [torch.empty((L, B, Hq, D), dtype=torch.float16, device="cuda") for _ in range(nbuf)]
    p2p = head and world > 1 and args.gather == "p2p"
    gathered = torch.empty((L, world, B, Hq, D), dtype=torch.float16, device="cuda") \
        if head and not p2p else None
    slice_bytes = B * Hq * D * 2
    if p2p:  # NVLink peer stores from the decode epilogue + epoch flags
        TD.connect_peer_gather(cache, L * world * slice_bytes)
        gptr, _ = cache.peer_buffer()
        torch.cuda.synchronize()
        barrier(world)  # ranks enter the GPU-side flag waits together
    epoch = [0]
    scale = 1.0 / math.sqrt(D)
    cur = list(lens)

    layer_flow = args.flow == "layer"

    def append_step(b):
        if not layer_flow:  # one fused append of every layer's new token
            cache.append_kv_all_layers(sids, knew[b].data_ptr(), vnew[b].data_ptr(), sp)

    def decode(b, l):
        if layer_flow:  # TransformerLayer::attention: this layer's append, then decode (RoPE on Q)
            cache.attention_step(l, q[b][l].data_ptr(), knew[b][l].data_ptr(), vnew[b][l].data_ptr(),
                                 out[b][l].data_ptr(), sids, scale, sp)
        elif p2p:  # decode + publish + pull of the other ranks' slices, fused
            epoch[0] += 1
            cache.decode_attention_peer(l, q[b][l].data_ptr(), sids, l * world * slice_bytes,
                                        epoch[0], scale, sp)
        else:
            cache.decode_attention(l, q[b][l].data_ptr(), out[b][l].data_ptr(), sids, scale, sp)

    def after_decode(b, l):
        if head and world > 1 and not p2p:  # the layer's outputs, all heads, on every rank
            TD.gather_head_outputs(out[b][l], gathered[l])

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kv_total = 0
    launches0 = None
    clocks = None
    sampler = None

    def run_step(i, events=None):
        nonlocal cur
        b = i % nbuf
        append_step(b)
        attended = [c + 1 for c in cur]
        for l in range(L):
            if events is not None:
                events[l][0].record(stream)
            decode(b, l)
            if events is not None:
                events[l][1].record(stream)
            after_decode(b, l)
        for s in sids:
            cache.advance_seq_len(s, 1)
        cur = attended
        return attended

    # timed steps: no events between the layers (an event between two
    # kernels would stop the next one from launching early)
    for i in range(steps):
        if i == args.warmup:
            torch.cuda.synchronize()
            sampler = ClockSampler(local)
            time.sleep(0.3)
            barrier(world)  # after the sampler starts: ranks enter the timed steps together
            launches0 = cache.pool_stats().kernel_launches
            start.record(stream)
        attended = run_step(i)
        if i >= args.warmup:
            kv_total += kv_bytes(attended, kcfg)
    end.record(stream)
    end.synchronize()
    launches = cache.pool_stats().kernel_launches - launches0
    if sampler:
        clocks = sampler.stop()
    ms = start.elapsed_time(end)
    cache.sync_check(sp)

    # roofline pass: the same steps again, with CUDA events around every
    # layer's decode call (decode + in-kernel merge) on the launching stream
    dec_ms, dec_bytes = 0.0, 0
    for i in range(args.steps):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(L)]
        attended = run_step(steps + i, evs)
        dec_bytes += kv_bytes(attended, kcfg) + 2 * L * B * Hq * D * 2 + \
            sum(-(-s // bs) for s in attended) * 4 * L
        torch.cuda.synchronize()
        dec_ms += sum(a.elapsed_time(z) for a, z in evs)
    cache.sync_check(sp)

    # ---- e2e: host buffers, H2D of each step's inputs and D2H of its output
    hk = torch.empty((nbuf, L, B, Hkv, D), dtype=torch.float16, pin_memory=True)
    hv = torch.empty_like(hk)
    hq = torch.empty((nbuf, L, B, Hq, D), dtype=torch.float16, pin_memory=True)
    oshape = (L, world, B, Hq, D) if head and world > 1 else (L, B, Hq, D)
    ho = torch.empty((nbuf,) + oshape, dtype=torch.float16, pin_memory=True)
    rt = C.CDLL("libcudart.so.12")  # the runtime torch loaded (same context)
    rt.cudaMemcpyAsync.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int, C.c_void_p]
    hk.copy_(torch.stack(knew).cpu())
    hv.copy_(torch.stack(vnew).cpu())
    hq.copy_(torch.stack(q).cpu())
    copy = torch.cuda.Stream()
    h2d_done = [torch.cuda.Event() for _ in range(nbuf)]
    comp_done = [torch.cuda.Event() for _ in range(nbuf)]
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def h2d(j):
        bb = j % nbuf
        with torch.cuda.stream(copy):
            if j >= nbuf:  # buffer bb was last read by step j - nbuf
                copy.wait_event(comp_done[bb])
            knew[bb].copy_(hk[bb], non_blocking=True)
            vnew[bb].copy_(hv[bb], non_blocking=True)
            q[bb].copy_(hq[bb], non_blocking=True)
            h2d_done[bb].record(copy)

    def e2e_loop(n, account):
        nonlocal cur
        kvb = 0
        h2d(0)
        for i in range(n):
            b = i % nbuf
            stream.wait_event(h2d_done[b])
            append_step(b)
            attended = [c + 1 for c in cur]
            for l in range(L):
                decode(b, l)
                after_decode(b, l)
            comp_done[b].record(stream)
            for s in sids:
                cache.advance_seq_len(s, 1)
            cur = attended
            if i + 1 < n:
                h2d(i + 1)  # the next step's inputs cross PCIe under this step's kernels
            with torch.cuda.stream(copy):
                copy.wait_event(comp_done[b])
                if p2p:  # the step's result is the gathered outputs of every layer
                    rt.cudaMemcpyAsync(ho[b].data_ptr(), gptr, ho[b].numel() * 2, 2, copy.cuda_stream)
                else:
                    ho[b].copy_(out[b] if gathered is None else gathered, non_blocking=True)
            if account:
                kvb += kv_bytes(attended, kcfg)
        return kvb

    torch.cuda.synchronize()
    barrier(world)
    e2e_loop(args.warmup, False)
    torch.cuda.synchronize()
    barrier(world)
    e_start.record(copy)
    e2e_kv = e2e_loop(args.steps, True)
    e_end.record(copy)
    e_end.synchronize()
    torch.cuda.synchronize()
    e2e_ms = e_start.elapsed_time(e_end)
    cache.sync_check(sp)

    res = dict(ms=ms, kv=kv_total, dec_ms=dec_ms, dec_bytes=dec_bytes,
               dec_launches=L * args.steps, launches=launches, clocks=clocks,
               e2e_ms=e2e_ms, e2e_kv=e2e_kv,
               h2d=(hk[0].numel() + hv[0].numel() + hq[0].numel()) * 2,
               d2h=ho[0].numel() * 2, B=B, global_b=global_b, lens=lens)
    cache.close()
    return res


# ------------------------------------------------------------ churn (c5) --

def run_churn(cfg, args, world, rank, local):
    """Config 5: a continuous-batching schedule over args.warmup + args.steps
    steps. Prompt prefill (per-layer appends) is timed apart from the decode
    step (fused append + decode attention of every layer + advance), which
    is what value / us_per_step measure."""
    import torch
    import tiny_llm_b200 as T
    from tiny_llm_b200.churn import ChurnSchedule

    L, Hq, Hkv, D, bs = cfg["L"], cfg["Hq"], cfg["Hkv"], cfg["D"], cfg["bs"]
    max_active, max_len = 256, 6144
    nblocks = ChurnSchedule.pool_blocks_for(max_active, 32, 4096, 256, bs, occupancy=0.8)
    cache = T.KVCache(num_layers=L, num_kv_heads=Hkv, head_dim=D, max_seq_len=max_len,
                      max_batch_size=max_active, block_size=bs, num_blocks=nblocks, num_q_heads=Hq,
                      rope_on_append=True, device=local)
    cache.permute_free_blocks(args.seed + rank)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    g = torch.Generator(device="cuda").manual_seed(args.seed * 7919 + rank)
    prompt_kv = torch.randn((2, 4096, Hkv, D), dtype=torch.float16, device="cuda", generator=g)
    step_k = torch.randn((L * max_active * Hkv * D,), dtype=torch.float16, device="cuda", generator=g)
    step_v = torch.randn_like(step_k)
    qbuf = torch.randn((L * max_active * Hq * D,), dtype=torch.float16, device="cuda", generator=g)
    obuf = torch.empty_like(qbuf)
    scale = 1.0 / math.sqrt(D)
    sch = ChurnSchedule(seed=args.seed + rank, rate=4.0, max_active=max_active, block_size=bs)
    ev_pairs, pf_pairs = [], []
    timing = [False]

    def prefill(sid, n):
        if timing[0]:
            a = torch.cuda.Event(enable_timing=True); a.record(stream); pf_pairs.append([a, None])
        for l in range(L):
            cache.append_kv(sid, l, prompt_kv[0].data_ptr(), prompt_kv[1].data_ptr(), n, sp)
        cache.advance_seq_len(sid, n)
        if timing[0]:
            z = torch.cuda.Event(enable_timing=True); z.record(stream); pf_pairs[-1][1] = z

    def decode_step(batch):
        B = len(batch)
        if timing[0]:
            a = torch.cuda.Event(enable_timing=True); a.record(stream)
        cache.append_kv_all_layers(batch, step_k.data_ptr(), step_v.data_ptr(), sp)
        qv = qbuf[: L * B * Hq * D].view(L, B, Hq, D)
        ov = obuf[: L * B * Hq * D].view(L, B, Hq, D)
        for l in range(L):
            cache.decode_attention(l, qv[l].data_ptr(), ov[l].data_ptr(), batch, scale, sp)
        for s in batch:
            cache.advance_seq_len(s, 1)
        if timing[0]:
            z = torch.cuda.Event(enable_timing=True); z.record(stream); ev_pairs.append((a, z))

    kv_total = 0
    sampler = None
    for i in range(args.warmup + args.steps):
        if i == args.warmup:
            torch.cuda.synchronize()
            sampler = ClockSampler(local)
            time.sleep(0.3)
            barrier(world)
            timing[0] = True
            launches0 = cache.pool_stats().kernel_launches
            occ0, act0, steps0 = sch.stats.occupancy_sum, sch.stats.active_sum, sch.stats.steps
        batch, attended = sch.step(cache, prefill, decode_step, max_len)
        if timing[0]:
            kv_total += sum(attended) * L * 2 * Hkv * D * 2
    torch.cuda.synchronize()
    clocks = sampler.stop() if sampler else None
    dec_ms = sum(a.elapsed_time(z) for a, z in ev_pairs)
    pf_ms = sum(a.elapsed_time(z) for a, z in pf_pairs)
    launches = cache.pool_stats().kernel_launches - launches0
    cache.sync_check(sp)
    n = sch.stats.steps - steps0
    res = dict(ms=dec_ms, kv=kv_total, prefill_ms=pf_ms, clocks=clocks, launches=launches,
               mean_active=(sch.stats.active_sum - act0) / n,
               occupancy=(sch.stats.occupancy_sum - occ0) / n,
               admitted=sch.stats.admitted, released=sch.stats.released,
               preempted=sch.stats.preempted, pool_blocks=nblocks)
    cache.close()
    return res


# -------------------------------------------------------- prefill (pf) ----

def run_prefill(cfg, args, world, rank, local):
    """A step = every prompt's K/V appended to every layer (tl_append_kv) and
    the causal prefill attention of every layer (tl_prefill_attention) over
    fresh sequences, which are released afterwards. value = causal attention
    FLOPs (4 * Hq * D per (query, key) pair with key <= query) per second."""
    import torch
    import tiny_llm_b200 as T
    L, Hq, Hkv, D, bs = cfg["L"], cfg["Hq"], cfg["Hkv"], cfg["D"], cfg["bs"]
    lens = list(cfg["lens"])
    B, n = len(lens), max(lens)
    cache = T.KVCache(num_layers=L, num_kv_heads=Hkv, head_dim=D, max_seq_len=n, max_batch_size=B,
                      block_size=bs, num_q_heads=Hq, rope_on_append=cfg["rope"], rope_theta=10000.0,
                      device=local)
    cache.permute_free_blocks(args.seed + rank)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    gen = torch.Generator(device="cuda")
    gen.manual_seed(args.seed * 7919 + rank)
    k = torch.randn((L, B, n, Hkv, D), dtype=torch.float16, device="cuda", generator=gen)
    v = torch.randn((L, B, n, Hkv, D), dtype=torch.float16, device="cuda", generator=gen)
    q = torch.randn((L, B * n, Hq, D), dtype=torch.float16, device="cuda", generator=gen)
    o = torch.empty_like(q)
    scale = 1.0 / math.sqrt(D)
    flops = L * B * 4 * Hq * D * (n * (n + 1) // 2)
    pairs = [None]

    def step(events=None):
        sids = [cache.allocate_sequence(n) for _ in range(B)]
        for l in range(L):
            for b, sid in enumerate(sids):
                cache.append_kv(sid, l, k[l, b].data_ptr(), v[l, b].data_ptr(), n, sp)
            if events is not None:
                events[l][0].record(stream)
            cache.prefill_attention(l, q[l].data_ptr(), o[l].data_ptr(), sids, [n] * B, scale, sp)
            if events is not None:
                events[l][1].record(stream)
        for sid in sids:
            cache.release_sequence(sid)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    time.sleep(0.3)
    barrier(world)
    launches0 = cache.pool_stats().kernel_launches
    a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        step()
    z.record(stream)
    z.synchronize()
    clocks = sampler.stop()
    ms = a.elapsed_time(z)
    launches = cache.pool_stats().kernel_launches - launches0
    cache.sync_check(sp)
    # roofline pass: events around each layer's prefill launch
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
    step(evs)
    torch.cuda.synchronize()
    pf_ms = sum(x.elapsed_time(y) for x, y in evs)
    # e2e: each step's Q/K/V from pinned host memory, outputs back to the host
    hq = torch.empty(q.shape, dtype=torch.float16, pin_memory=True)
    hk = torch.empty(k.shape, dtype=torch.float16, pin_memory=True)
    hv = torch.empty(v.shape, dtype=torch.float16, pin_memory=True)
    ho = torch.empty(o.shape, dtype=torch.float16, pin_memory=True)
    hq.copy_(q.cpu()); hk.copy_(k.cpu()); hv.copy_(v.cpu())
    torch.cuda.synchronize()
    barrier(world)
    ea, ez = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ea.record(stream)
    for _ in range(args.steps):
        q.copy_(hq, non_blocking=True)
        k.copy_(hk, non_blocking=True)
        v.copy_(hv, non_blocking=True)
        step()
        ho.copy_(o, non_blocking=True)
    ez.record(stream)
    ez.synchronize()
    e2e_ms = ea.elapsed_time(ez)
    cache.sync_check(sp)
    cache.close()
    return dict(ms=ms, flops=flops * args.steps, pf_ms=pf_ms, pf_flops=flops, e2e_ms=e2e_ms,
                h2d=(hq.numel() + hk.numel() + hv.numel()) * 2, d2h=ho.numel() * 2,
                launches=launches, clocks=clocks, B=B, n=n)


def _qkv_weights(cfg, L, gen):
    import torch
    hidden, group, Hq, Hkv, D = cfg["hidden"], cfg["group"], cfg["Hq"], cfg["Hkv"], cfg["D"]
    ws = []
    for _ in range(L):
        layer = []
        for n in (Hq * D, Hkv * D, Hkv * D):
            w = torch.randint(-127, 128, (hidden, n), dtype=torch.int8, device="cuda", generator=gen)
            sc = (torch.rand((hidden // group, n), device="cuda", generator=gen) * 0.018 + 0.002).half()
            layer += [w, sc]
        ws.append(layer)
    return ws


def qkv_weight_bytes(cfg):
    hidden, group, Hq, Hkv, D = cfg["hidden"], cfg["group"], cfg["Hq"], cfg["Hkv"], cfg["D"]
    n = (Hq + 2 * Hkv) * D
    return hidden * n + (hidden // group) * n * 2


def run_qkv(cfg, args, world, rank, local):
    """A step = the decode step's Q/K/V projections of every layer for B
    sequences, one token each, with K/V written into the cache at each
    sequence's length and Q rotated (tl_project_qkv_append). value = weight
    bytes (int8 + fp16 scales) streamed per second; the activations, Q and
    the K/V rows are small beside them."""
    import torch
    import tiny_llm_b200 as T
    L, Hq, Hkv, D, bs = cfg["L"], cfg["Hq"], cfg["Hkv"], cfg["D"], cfg["bs"]
    hidden, group = cfg["hidden"], cfg["group"]
    lens = list(cfg["lens"])
    B, P = len(lens), max(lens)
    cache = T.KVCache(num_layers=L, num_kv_heads=Hkv, head_dim=D, max_seq_len=P + 8, max_batch_size=B,
                      block_size=bs, num_q_heads=Hq, rope_on_append=cfg["rope"], rope_theta=10000.0,
                      device=local)
    cache.permute_free_blocks(args.seed + rank)
    sids = [cache.allocate_sequence(P + 8) for _ in range(B)]
    for sid in sids:
        cache.reserve(sid, P + 1)
        cache.advance_seq_len(sid, P)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    gen = torch.Generator(device="cuda")
    gen.manual_seed(args.seed * 7919 + rank)
    ws = _qkv_weights(cfg, L, gen)
    packed = args.qkv_weights == "packed"
    if packed:  # once, as at model load: the tile-blocked copy replaces the row-major one
        for layer in ws:
            for j in (0, 2, 4):
                pk = torch.empty_like(layer[j])
                T.pack_qkv_weight(layer[j].data_ptr(), hidden, layer[j].shape[1], pk.data_ptr(), sp)
                layer[j] = pk
        torch.cuda.synchronize()
    project = cache.project_qkv_append_packed if packed else cache.project_qkv_append
    x = torch.randn((L, B, hidden), dtype=torch.float16, device="cuda", generator=gen)
    q = torch.empty((L, B, Hq * D), dtype=torch.float16, device="cuda")

    def step(s=None):
        s = s or sp
        for l in range(L):
            w = ws[l]
            project(l, x[l].data_ptr(), hidden, w[0].data_ptr(), w[1].data_ptr(), w[2].data_ptr(),
                    w[3].data_ptr(), w[4].data_ptr(), w[5].data_ptr(), group, sids, q[l].data_ptr(), s)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    time.sleep(0.3)
    barrier(world)
    launches0 = cache.pool_stats().kernel_launches
    a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        step()
    z.record(stream)
    z.synchronize()
    clocks = sampler.stop()
    ms = a.elapsed_time(z)
    launches = cache.pool_stats().kernel_launches - launches0
    cache.sync_check(sp)
    # roofline pass: one step's L launches captured in a CUDA graph and
    # replayed (the positions are fixed and the op rewrites the same rows),
    # so the time is the kernels' own, without the host's per-call work
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step(torch.cuda.current_stream().cuda_stream)
    for _ in range(3):
        graph.replay()
    reps = 10
    ga, gz = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ga.record(stream)
    for _ in range(reps):
        graph.replay()
    gz.record(stream)
    gz.synchronize()
    k_ms = ga.elapsed_time(gz) / (reps * L)
    del graph
    cache.sync_check(sp)
    # e2e: each step's activations from pinned host memory, Q back to the host
    hx = torch.empty(x.shape, dtype=torch.float16, pin_memory=True)
    hq = torch.empty(q.shape, dtype=torch.float16, pin_memory=True)
    hx.copy_(x.cpu())
    torch.cuda.synchronize()
    barrier(world)
    ea, ez = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ea.record(stream)
    for _ in range(args.steps):
        x.copy_(hx, non_blocking=True)
        step()
        hq.copy_(q, non_blocking=True)
    ez.record(stream)
    ez.synchronize()
    e2e_ms = ea.elapsed_time(ez)
    cache.sync_check(sp)
    # CPU baseline: the oracle's restatement of the reference matmul (fp32,
    # OpenMP) on one layer's three projections for every row
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        import numpy as np
        import oracle as O
        xs = x[0].cpu().numpy().view(np.uint16)
        cw = [(torch.randint(-127, 128, (hidden, n), dtype=torch.int8).numpy(),
               ws[0][2 * j + 1].cpu().numpy().view(np.uint16)) for j, n in enumerate((Hq * D, Hkv * D, Hkv * D))]
        t0 = time.perf_counter()
        for w, sc in cw:
            O.w8a16_matmul(xs, w, sc, group)
        el = time.perf_counter() - t0
        cpu = {"value": round(qkv_weight_bytes(cfg) / el / 1e9, 3), "unit": "GB/s",
               "cores": os.cpu_count() or 1, "kind": "port",
               "sample": f"one layer's Q/K/V projections for all {B} rows (oracle fp32 restatement of "
                         "kernels::w8a16_matmul, OpenMP), the K/V append not included"}
    cache.close()
    wb = qkv_weight_bytes(cfg)
    io = B * hidden * 2 + B * Hq * D * 2 + 2 * B * Hkv * D * 2
    return dict(ms=ms, bytes=(wb + io) * L * args.steps, wbytes=wb * L * args.steps, k_ms=k_ms,
                graph_ms_per_step=k_ms * L,
                k_bytes=wb + io, e2e_ms=e2e_ms, h2d=hx.numel() * 2, d2h=hq.numel() * 2,
                launches=launches, clocks=clocks, B=B, cpu=cpu)


def run_sampling(cfg, args, world, rank, local):
    """A step = one tl_sample_tokens launch over B rows of logits (a new
    uniform per step). value = tokens sampled per second."""
    import torch
    import tiny_llm_b200 as T
    B, V = len(cfg["lens"]), cfg["vocab"]
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    gen = torch.Generator(device="cuda")
    gen.manual_seed(args.seed * 7919 + rank)
    lg = (torch.randn((B, V), device="cuda", generator=gen) * 3).half()
    tok = torch.empty(B, dtype=torch.int32, device="cuda")
    kw = dict(do_sample=True, temperature=0.8, top_k=50, top_p=0.9)

    def step(i):
        T.sample_tokens(lg.data_ptr(), V, B, V, tok.data_ptr(), seed=args.seed + rank, step=i, stream=sp, **kw)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    time.sleep(0.3)
    barrier(world)
    a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(args.steps):
        step(args.warmup + i)
    z.record(stream)
    z.synchronize()
    clocks = sampler.stop()
    ms = a.elapsed_time(z)
    hl = torch.empty(lg.shape, dtype=torch.float16, pin_memory=True)
    ht = torch.empty(tok.shape, dtype=torch.int32, pin_memory=True)
    hl.copy_(lg.cpu())
    torch.cuda.synchronize()
    ea, ez = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ea.record(stream)
    for i in range(args.steps):
        lg.copy_(hl, non_blocking=True)
        step(i)
        ht.copy_(tok, non_blocking=True)
    ez.record(stream)
    ez.synchronize()
    e2e_ms = ea.elapsed_time(ez)
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        import numpy as np
        import oracle as O
        sys.path.insert(0, str(ROOT / "oracle"))
        import sampling as S
        rows = O.f16_to_f32(lg[:4].cpu().numpy().view(np.uint16)).astype(np.float64)
        t0 = time.perf_counter()
        for r in range(rows.shape[0]):
            S.sample(rows[r], seed=args.seed, step=0, row=r, **kw)
        el = time.perf_counter() - t0
        cpu = {"value": round(rows.shape[0] / el, 2), "unit": "tokens/s", "cores": 1, "kind": "port",
               "sample": "4 rows through the oracle's float64 restatement of the reference's top-p sampler (numpy sort per row)"}
    return dict(ms=ms, tokens=B * args.steps, e2e_ms=e2e_ms, h2d=hl.numel() * 2, d2h=ht.numel() * 4,
                clocks=clocks, B=B, V=V, cpu=cpu, launches=args.steps)


def run_reference_qkv(cfg, args, world, rank, local):
    """The reference's own decode-step projections and append, unchanged:
    three kernels::w8a16_matmul per layer into q/k/v buffers (given all B
    rows at once, which the reference engine never does) and
    KVCacheManager::appendKV of each sequence's row. No RoPE (the reference
    has none)."""
    import torch
    lib, why = load_ref()
    if lib is None:
        return None, why
    L, Hq, Hkv, D = cfg["L"], cfg["Hq"], cfg["Hkv"], cfg["D"]
    hidden, group = cfg["hidden"], cfg["group"]
    B, P = len(cfg["lens"]), max(cfg["lens"])
    h = C.c_void_p()
    if lib.ref_kv_create(L, Hkv, D, P + 8, B, C.byref(h)) != 0:
        return None, "reference KVCacheManager::create failed: " + lib.ref_last_error().decode()
    sids = []
    for _ in range(B):
        sid = C.c_int()
        assert lib.ref_kv_allocate(h, P + 8, C.byref(sid)) == 0
        assert lib.ref_kv_advance(h, sid.value, P) == 0
        sids.append(sid.value)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    gen = torch.Generator(device="cuda")
    gen.manual_seed(args.seed * 7919 + rank)
    ws = _qkv_weights(cfg, L, gen)
    x = torch.randn((L, B, hidden), dtype=torch.float16, device="cuda", generator=gen)
    q = torch.empty((L, B, Hq * D), dtype=torch.float16, device="cuda")
    kb = torch.empty((B, Hkv * D), dtype=torch.float16, device="cuda")
    vb = torch.empty_like(kb)
    row = Hkv * D * 2

    def step():
        for l in range(L):
            w = ws[l]
            for out, j, n in ((q[l], 0, Hq * D), (kb, 1, Hkv * D), (vb, 2, Hkv * D)):
                rc = lib.ref_w8a16_matmul(x[l].data_ptr(), w[2 * j].data_ptr(), w[2 * j + 1].data_ptr(),
                                          out.data_ptr(), B, n, hidden, group, sp)
                assert rc == 0, lib.ref_last_error().decode()
            for b, sid in enumerate(sids):
                rc = lib.ref_kv_append(h, sid, l, kb.data_ptr() + b * row, vb.data_ptr() + b * row, 1, sp)
                assert rc == 0, lib.ref_last_error().decode()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    time.sleep(0.3)
    a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        step()
    z.record(stream)
    z.synchronize()
    clocks = sampler.stop()
    ms = a.elapsed_time(z)
    hx = torch.empty(x.shape, dtype=torch.float16, pin_memory=True)
    hq = torch.empty(q.shape, dtype=torch.float16, pin_memory=True)
    hx.copy_(x.cpu())
    torch.cuda.synchronize()
    ea, ez = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ea.record(stream)
    for _ in range(args.steps):
        x.copy_(hx, non_blocking=True)
        step()
        hq.copy_(q, non_blocking=True)
    ez.record(stream)
    ez.synchronize()
    e2e_ms = ea.elapsed_time(ez)
    lib.ref_kv_destroy(h)
    wb = qkv_weight_bytes(cfg) * L * args.steps
    return dict(ms=ms, wbytes=wb, e2e_ms=e2e_ms, h2d=hx.numel() * 2, d2h=hq.numel() * 2, clocks=clocks,
                B=B), None


# ---------------------------------------------------------- reference path --

def load_ref():
    p = ROOT / "oracle" / "_ref" / "libtllm_ref.so"
    if not p.exists():
        return None, f"{p.relative_to(ROOT)} was not built (needs the reference sources at build time)"
    lib = C.CDLL(str(p))
    vp, i, f = C.c_void_p, C.c_int, C.c_float
    lib.ref_kv_create.argtypes = [i, i, i, i, i, C.POINTER(vp)]
    lib.ref_kv_allocate.argtypes = [vp, i, C.POINTER(i)]
    lib.ref_kv_append.argtypes = [vp, i, i, vp, vp, i, vp]
    lib.ref_kv_advance.argtypes = [vp, i, i]
    lib.ref_kv_destroy.argtypes = [vp]
    lib.ref_attention_decode.argtypes = [vp, vp, vp, vp, f, i, i, i, i, vp]
    if hasattr(lib, "ref_w8a16_matmul"):
        lib.ref_w8a16_matmul.argtypes = [vp, vp, vp, vp, i, i, i, i, vp]
    lib.ref_last_error.restype = C.c_char_p
    return lib, None


def run_reference(cfg, args, world, rank, local):
    """The reference's own path, unchanged: KVCacheManager::appendKV per
    (sequence, layer) and kernels::attention_decode per layer. The kernel
    reads [B][H][S][D] K/V (attention.cu:23-25), so it is given per-query-head
    (GQA-expanded) buffers of that layout; its append writes the manager's
    contiguous slots. Uniform-length configs only (one launch per layer)."""
    import torch

    lib, why = load_ref()
    if lib is None:
        return None, why
    L, Hq, Hkv, D = cfg["L"], cfg["Hq"], cfg["Hkv"], cfg["D"]
    lens, global_b = rank_lens(cfg, args, world, rank)
    if len(set(lens)) != 1:
        return None, "reference arm runs uniform-length configs only (one attention_decode per layer)"
    B, P = len(lens), lens[0]
    steps = args.warmup + args.steps
    if P + 2 * steps + 2 > 12256:
        return None, ("reference kernels::attention_decode cannot launch above context 12256 "
                      "(dynamic smem (S+32)*4 B > 48 KiB, kernels/attention.cu:124)")
    max_len = P + 2 * steps + 2
    h = C.c_void_p()
    if lib.ref_kv_create(L, Hkv, D, max_len, B, C.byref(h)) != 0:
        return None, "reference KVCacheManager::create failed: " + lib.ref_last_error().decode()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(args.seed * 7919 + rank)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    sids = []
    for _ in range(B):
        sid = C.c_int()
        assert lib.ref_kv_allocate(h, max_len, C.byref(sid)) == 0
        sids.append(sid.value)
    for sid in sids:
        for l in range(L):
            kv = torch.randn((2, P, Hkv, D), dtype=torch.float16, device="cuda", generator=gen)
            assert lib.ref_kv_append(h, sid, l, kv[0].data_ptr(), kv[1].data_ptr(), P, sp) == 0
        lib.ref_kv_advance(h, sid, P)
    # Attention inputs in the kernel's [B][Hq][S][D] layout, per layer.
    Kd = [torch.randn((B, Hq, max_len, D), dtype=torch.float16, device="cuda", generator=gen) for _ in range(L)]
    Vd = [torch.randn((B, Hq, max_len, D), dtype=torch.float16, device="cuda", generator=gen) for _ in range(L)]
    knew = torch.randn((L, B, Hkv, D), dtype=torch.float16, device="cuda", generator=gen)
    vnew = torch.randn((L, B, Hkv, D), dtype=torch.float16, device="cuda", generator=gen)
    q = torch.randn((L, B, Hq, D), dtype=torch.float16, device="cuda", generator=gen)
    out = torch.empty((L, B, Hq, D), dtype=torch.float16, device="cuda")
    scale = 1.0 / math.sqrt(D)

    def step(cur, timed_events=None):
        for bi, sid in enumerate(sids):
            for l in range(L):
                rc = lib.ref_kv_append(h, sid, l, knew[l, bi].data_ptr(), vnew[l, bi].data_ptr(), 1, sp)
                assert rc == 0, lib.ref_last_error().decode()
        S = cur + 1
        for l in range(L):
            if timed_events is not None:
                timed_events[l][0].record(stream)
            rc = lib.ref_attention_decode(q[l].data_ptr(), Kd[l].data_ptr(), Vd[l].data_ptr(),
                                          out[l].data_ptr(), scale, B, Hq, S, D, sp)
            assert rc == 0, lib.ref_last_error().decode()
            if timed_events is not None:
                timed_events[l][1].record(stream)
        for sid in sids:
            lib.ref_kv_advance(h, sid, 1)
        return S

    cur = P
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kv_total = 0
    sampler = None
    all_evs = []
    for i in range(steps):
        if i == args.warmup:
            torch.cuda.synchronize()
            sampler = ClockSampler(local)
            time.sleep(0.3)
            barrier(world)
            start.record(stream)
        evs = None
        if i >= args.warmup:
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(L)]
            all_evs += evs
        S = step(cur, evs)
        if evs:
            kv_total += S * B * L * 2 * Hkv * D * 2
        cur = S
    end.record(stream)
    end.synchronize()
    ms = start.elapsed_time(end)
    dec_ms = sum(a.elapsed_time(z) for a, z in all_evs)
    clocks = sampler.stop() if sampler else None

    # e2e: pinned host inputs copied in each step, outputs copied back.
    hk = knew.cpu().pin_memory()
    hv = vnew.cpu().pin_memory()
    hq = q.cpu().pin_memory()
    ho = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_kv = 0
    for i in range(steps):
        if i == args.warmup:
            torch.cuda.synchronize()
            barrier(world)
            e_start.record(stream)
        knew.copy_(hk, non_blocking=True)
        vnew.copy_(hv, non_blocking=True)
        q.copy_(hq, non_blocking=True)
        S = step(cur)
        ho.copy_(out, non_blocking=True)
        if i >= args.warmup:
            e2e_kv += S * B * L * 2 * Hkv * D * 2
        cur = S
    e_end.record(stream)
    e_end.synchronize()
    e2e_ms = e_start.elapsed_time(e_end)
    lib.ref_kv_destroy(h)
    return dict(ms=ms, kv=kv_total, dec_ms=dec_ms, clocks=clocks, e2e_ms=e2e_ms, e2e_kv=e2e_kv,
                h2d=(hk.numel() + hv.numel() + hq.numel()) * 2, d2h=ho.numel() * 2, B=B,
                global_b=global_b), None


# ------------------------------------------------------------ CPU baseline --

def cpu_baseline(cfg, seed, budget_s=10.0):
    """The oracle's fp32 decode (reference kernel math, OpenMP over
    (sequence, kv_head)) on a bounded sample of the workload: 4 sequences of
    one layer at the config's context, repeated for ~budget_s seconds."""
    import numpy as np
    import oracle as O

    D, Hkv, Hq, bs = cfg["D"], cfg["Hkv"], cfg["Hq"], cfg["bs"]
    S = min(seq_lens(cfg, seed, 0)[0] + 1, 8193)
    Bs = 4
    nb_seq = -(-S // bs)
    g = O.geom(1, Hkv, D, bs, Bs * nb_seq)
    pool = O.normal_f16((2 * Bs * nb_seq * bs * Hkv * D,), seed + 17)
    bt = np.arange(Bs * nb_seq, dtype=np.int32).reshape(Bs, nb_seq)
    lens = np.full(Bs, S, np.int32)
    q = O.normal_f16((Bs, Hq, D), seed + 18)
    threads = len(os.sched_getaffinity(0))
    t0 = time.perf_counter()
    reps = 0
    while True:
        _, used = O.decode_paged_f32(pool, g, 0, bt, lens, q, Hq, 1.0 / math.sqrt(D), threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    kv = reps * Bs * S * 2 * Hkv * D * 2
    return {"value": round(kv / el / 1e9, 3), "unit": "GB/s", "cores": used, "kind": "port",
            "sample": f"{reps} x (1 layer, {Bs} seqs x {S} tokens, Hq={Hq} Hkv={Hkv} D={D}) "
                      f"fp32 oracle decode in {el:.1f}s on {threads} host threads"}


def cpu_baseline_prefill(cfg, seed, budget_s=10.0):
    """The oracle's fp32 attention (reference kernel math, OpenMP) on a
    bounded sample of the prefill workload: query rows of one 4096-token
    prompt of one layer, every 64th position (so the rows' mean causal length
    is the prompt's), each attending the cached tokens up to its position,
    repeated for ~budget_s seconds. value = causal attention FLOPs per
    second, counted as the GPU arm counts them."""
    import numpy as np
    import oracle as O

    D, Hkv, Hq, bs = cfg["D"], cfg["Hkv"], cfg["Hq"], cfg["bs"]
    n = max(cfg["lens"])
    nb = -(-n // bs)
    g = O.geom(1, Hkv, D, bs, nb)
    pool = O.normal_f16((2 * nb * bs * Hkv * D,), seed + 27)
    pos = np.arange(32, n, 64, dtype=np.int32)  # mid-points of 64-row groups
    R = len(pos)
    bt = np.tile(np.arange(nb, dtype=np.int32), (R, 1))
    lens = pos + 1
    q = O.normal_f16((R, Hq, D), seed + 28)
    threads = len(os.sched_getaffinity(0))
    t0 = time.perf_counter()
    reps = 0
    while True:
        _, used = O.decode_paged_f32(pool, g, 0, bt, lens, q, Hq, 1.0 / math.sqrt(D), threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    flops = reps * 4 * Hq * D * int(lens.sum())
    return {"value": round(flops / el / 1e12, 6), "unit": "TFLOP/s", "cores": used, "kind": "port",
            "sample": f"{reps} x ({R} query rows of one {n}-token prompt, every 64th position, 1 layer, "
                      f"Hq={Hq} Hkv={Hkv} D={D}) fp32 oracle attention in {el:.1f}s on {threads} host threads"}


# ------------------------------------------------------------------- main --

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default 20; c5: 2000 scheduler steps)")
    ap.add_argument("--warmup", type=int, default=None,
                    help="untimed steps first (default 5; c5: 300, until the schedule is "
                         "at its steady state)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c2")
    ap.add_argument("--layout", choices=["token", "head"], default="token")
    ap.add_argument("--gather", choices=["p2p", "nccl"], default="p2p",
                    help="head-shard output exchange: fused into the decode call (each rank "
                         "publishes a flag, then pulls the other ranks' slices over NVLink), "
                         "or an NCCL all-gather after each layer")
    ap.add_argument("--shard", choices=["batch", "head"], default="batch",
                    help="multi-GPU split: whole sequences per rank, or KV heads per rank with "
                         "an all-gather of outputs each layer")
    ap.add_argument("--scaling", choices=["strong", "weak"], default="strong",
                    help="batch shard: strong splits the config's batch over the ranks (fixed "
                         "total work); weak gives every rank the whole batch")
    ap.add_argument("--flow", choices=["fused", "layer"], default="fused",
                    help="fused: one append of every layer's new token, then decode per layer; "
                         "layer: per layer, append that layer's token then decode with RoPE on Q "
                         "(the TransformerLayer::attention flow, tl_attention_step)")
    ap.add_argument("--qkv-weights", choices=["packed", "reference"], default="packed",
                    help="qkv config: weights repacked once by tl_qkv_pack_weight (tl_project_qkv_append_packed), "
                         "or read in the reference's QuantizedWeight layout (tl_project_qkv_append)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--layers", type=int, default=0,
                    help="override the config's layer count (small profiling cases; "
                         "every decode launch keeps the config's shape)")
    ap.add_argument("--cpu-baseline-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 2000 if args.config == "c5" else 20
    if args.warmup is None:
        args.warmup = 300 if args.config == "c5" else 5
    args.warmup = max(args.warmup, 3)
    cfg = dict(CONFIGS[args.config])
    if args.layers > 0:
        cfg["L"] = args.layers
        cfg["workload"] += f" [{args.layers} layers]"
    world, rank, local = dist_setup()
    peak, peak_kind = peaks()
    base_config = {"workload": cfg["workload"], "layers": cfg["L"], "q_heads": cfg["Hq"],
                   "kv_heads": cfg["Hkv"], "head_dim": cfg["D"], "block_size": cfg["bs"],
                   "rope_on_append": cfg["rope"], "layout": args.layout,
                   "parallelism": (f"head-shard x{world} (KV heads per GPU, outputs gathered per layer by "
                                   + ("a flag publish and NVLink pull fused into the decode call)"
                                      if args.gather == "p2p" else "NCCL all-gather)")
                                   if args.shard == "head" else
                                   f"batch-shard x{world} (" + ("the batch split over the GPUs by KV bytes"
                                                               if args.scaling == "strong" else
                                                               "a whole batch per GPU") +
                                   ", independent sequences, no collective)"),
                   "l2": "KV bytes per step far above the 126 MB L2; no flush needed",
                   "flow": ("per layer: append that layer's token, decode with RoPE on Q "
                            "(tl_attention_step)" if args.flow == "layer" else
                            "one fused append of all layers' tokens, then decode per layer"),
                   "seed": args.seed}
    if args.flow == "layer" and (args.shard == "head" or args.config == "c5" or args.impl == "reference"):
        raise SystemExit("--flow layer applies to the batch-sharded uniform/ragged configs of our arm")

    if args.impl == "reference":
        if args.config == "c5":
            res, why = None, ("reference arm runs uniform-length configs only; the reference "
                              "engine has no continuous batching (max_batch_size=1)")
        elif args.config == "pf":
            res, why = None, ("reference arm covers the decode configs; the reference prefill kernel "
                              "is compared in tests/test_gpu_reference.py")
        elif args.config == "smp":
            res, why = None, ("the reference samples on the host after a synchronize and a logits copy "
                              "(src/inference_engine.cpp:296-307) inside its engine; its samplers are restated "
                              "in oracle/sampling.py (the timed CPU baseline of our arm) and compared by "
                              "tests/test_gpu_sampling.py")
        elif args.config == "qkv":
            res, why = run_reference_qkv(cfg, args, world, rank, local)
            if res is not None:
                ms = barrier_max(res["ms"], world)
                wbt = barrier_sum(res["wbytes"], world)
                e2e_ms = barrier_max(res["e2e_ms"], world)
                if rank == 0:
                    value = wbt / (ms / 1e3) / 1e9
                    ev = wbt / (e2e_ms / 1e3) / 1e9
                    line = {"impl": "reference", "metric": "decode QKV projection + append, weight GB/s",
                            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
                            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                            "dtype": "int8 weights x f16 activations (fp32 accumulate)",
                            "data": "synthetic seeded int8 weights, fp16 scales and activations",
                            "config": dict(base_config, global_batch=res["B"] * world, hidden=cfg["hidden"],
                                           group_size=cfg["group"],
                                           layout="reference contiguous slots; three w8a16_matmul + appendKV per layer"),
                            "cpu_baseline": {"value": round(value, 2), "unit": "GB/s", "cores": 0,
                                             "kind": "reference",
                                             "sample": "the reference's own CUDA path (kernels::w8a16_matmul x3 + appendKV memcpys per layer) rebuilt for sm_100a, on the GPU: the reference has no host implementation of this path"},
                            "e2e": {"value": round(ev, 2), "unit": "GB/s", "h2d_bytes_per_step": res["h2d"],
                                    "d2h_bytes_per_step": res["d2h"]},
                            "clocks": res["clocks"]}
                    print(json.dumps(line), flush=True)
                if world > 1:
                    import torch.distributed as dist
                    dist.destroy_process_group()
                return
        else:
            res, why = run_reference(cfg, args, world, rank, local)
        if res is None:
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": why}), flush=True)
            if world > 1:
                import torch.distributed as dist
                dist.destroy_process_group()
            return
        ms = barrier_max(res["ms"], world)
        rank_ms = gather_values(res["ms"], world)
        kv = barrier_sum(res["kv"], world)
        e2e_ms = barrier_max(res["e2e_ms"], world)
        e2e_kv = barrier_sum(res["e2e_kv"], world)
        if rank == 0:
            value = kv / (ms / 1e3) / 1e9
            ev = e2e_kv / (e2e_ms / 1e3) / 1e9
            line = {"impl": "reference", "metric": "decode attn+append KV-read GB/s",
                    "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
                    "steps": args.steps, "warmup": args.warmup,
                    "ms_per_step": round(ms / args.steps, 4),
                    "us_per_step": round(1e3 * ms / args.steps, 1),
                    "per_rank_ms_per_step": [round(x / args.steps, 4) for x in rank_ms],
                    "higher_is_better": True, "scaling": args.scaling if world > 1 else "strong",
                    "vs_baseline": None,
                    "dtype": "f16 (fp32 accumulate)", "data": "synthetic N(0,1) fp16, seeded",
                    "config": dict(base_config, global_batch=res["global_b"], layout="reference contiguous slots + [B][H][S][D] kernel input"),
                    "cpu_baseline": {"value": round(value, 2), "unit": "GB/s", "cores": 0,
                                     "kind": "reference",
                                     "sample": "the reference's own CUDA path (appendKV memcpys + attention_decode) rebuilt for sm_100a, on the GPU: the reference has no host implementation of this path"},
                    "e2e": {"value": round(ev, 2), "unit": "GB/s",
                            "h2d_bytes_per_step": res["h2d"], "d2h_bytes_per_step": res["d2h"]},
                    "decode_kernel_gbs": round(kv / world / (res["dec_ms"] / 1e3) / 1e9, 1) if res["dec_ms"] else None,
                    "clocks": res["clocks"]}
            print(json.dumps(line), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    if args.config == "pf":
        res = run_prefill(cfg, args, world, rank, local)
        cpu = None
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline_prefill(cfg, args.seed, args.cpu_baseline_seconds)
        ms = barrier_max(res["ms"], world)
        fl = barrier_sum(res["flops"], world)
        e2e_ms = barrier_max(res["e2e_ms"], world)
        if rank == 0:
            pk = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
            tpeak = float(pk.get("bf16_tflops", 1590.0))
            achieved = res["pf_flops"] / (res["pf_ms"] / 1e3) / 1e12
            line = {"metric": "prefill attention TFLOP/s (causal)", "value": round(fl / (ms / 1e3) / 1e12, 2),
                    "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                    "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "weak",
                    "vs_baseline": None, "dtype": "f16 (fp32 accumulate)",
                    "data": "synthetic N(0,1) fp16 Q/K/V from a seeded generator (no dataset)",
                    "config": dict({k: v for k, v in base_config.items() if k not in ("l2", "flow")},
                                   global_batch=res["B"] * world, seq_len=res["n"],
                                   step="append every layer's prompt K/V, causal prefill per layer, release",
                                   l2="K/V of a layer (67 MB) kept in L2 across the query blocks; Q/O stream"),
                    "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": tpeak,
                                 "unit": "TFLOP/s", "frac": round(achieved / tpeak, 4),
                                 "traffic": launch_traffic("pf"),
                                 "kernel": "paged_prefill_tc_kernel (tcgen05.mma, TMEM accumulators)",
                                 "peak_source": "measured cuBLAS bf16 dense (MEASURED_PEAKS.json bf16_tflops)"
                                 if pk else "fallback"},
                    "cpu_baseline": cpu,
                    "e2e": {"value": round(fl / (e2e_ms / 1e3) / 1e12, 2), "unit": "TFLOP/s",
                            "h2d_bytes_per_step": res["h2d"], "d2h_bytes_per_step": res["d2h"]},
                    "clocks": res["clocks"], "gpu_launches": res["launches"]}
            print(json.dumps(line), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    if args.config == "smp":
        res = run_sampling(cfg, args, world, rank, local)
        ms = barrier_max(res["ms"], world)
        toks = barrier_sum(res["tokens"], world)
        e2e_ms = barrier_max(res["e2e_ms"], world)
        if rank == 0:
            per = ms / args.steps
            lbytes = res["B"] * res["V"] * 2
            achieved = lbytes / (per / 1e3) / 1e9
            line = {"metric": "next-token sampling tokens/s", "value": round(toks / (ms / 1e3), 1),
                    "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                    "ms_per_step": round(per, 4), "higher_is_better": True, "scaling": "weak",
                    "vs_baseline": None, "dtype": "f16 logits (fp32 softmax mass)",
                    "data": "synthetic N(0, 3) fp16 logits from a seeded generator",
                    "config": {"workload": cfg["workload"], "rows": res["B"] * world, "vocab": res["V"],
                               "strategy": "top-p 0.9, T 0.8 (do_sample)",
                               "l2": "8 MB of logits, re-read per pass from L2 (one read from HBM)"},
                    "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                                 "frac": round(achieved / peak, 4), "traffic": launch_traffic("smp"),
                                 "kernel": "sample_kernel (a cluster of 8 CTAs per row, the row's slice of keys in shared memory)",
                                 "note": "one HBM read of the logits; bound by ~10 cluster-wide histogram reductions per row, not by HBM",
                                 "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback"},
                    "cpu_baseline": res["cpu"],
                    "e2e": {"value": round(toks / (e2e_ms / 1e3), 1), "unit": "tokens/s",
                            "h2d_bytes_per_step": res["h2d"], "d2h_bytes_per_step": res["d2h"]},
                    "clocks": res["clocks"], "gpu_launches": res["launches"]}
            print(json.dumps(line), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    if args.config == "qkv":
        res = run_qkv(cfg, args, world, rank, local)
        ms = barrier_max(res["ms"], world)
        wbt = barrier_sum(res["wbytes"], world)
        e2e_ms = barrier_max(res["e2e_ms"], world)
        if rank == 0:
            achieved = res["k_bytes"] / (res["k_ms"] / 1e3) / 1e9
            line = {"metric": "decode QKV projection + append, weight GB/s", "value": round(wbt / (ms / 1e3) / 1e9, 2),
                    "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                    "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "weak",
                    "vs_baseline": None, "dtype": "int8 weights x f16 activations (fp32 accumulate)",
                    "data": "synthetic seeded int8 weights, fp16 scales and activations (no checkpoint)",
                    "config": dict({k: v for k, v in base_config.items() if k not in ("flow",)},
                                   global_batch=res["B"] * world, hidden=cfg["hidden"], group_size=cfg["group"],
                                   step="per layer: Q/K/V projections of every sequence's token, K/V into the pool, Q rotated",
                                   weights=("tile-blocked copies made once at setup by tl_qkv_pack_weight "
                                            "(tl_project_qkv_append_packed)" if args.qkv_weights == "packed" else
                                            "the reference's QuantizedWeight layout (tl_project_qkv_append)"),
                                   l2="839 MB of weights per step, each layer's read once; no flush needed"),
                    "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                                 "frac": round(achieved / peak, 4), "traffic": launch_traffic("qkv"),
                                 "algorithmic_bytes_per_launch": res["k_bytes"],
                                 "kernel": "qkv_append_tc_kernel (W8A16 on tcgen05, fp16 weights in TMEM, split-K, fused append)",
                                 "us_per_launch": round(res["k_ms"] * 1e3, 2),
                                 "timed_as": "the step's launches replayed from a CUDA graph (kernel time without host calls)",
                                 "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback"},
                    "cpu_baseline": res["cpu"],
                    "e2e": {"value": round(wbt / (e2e_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                            "h2d_bytes_per_step": res["h2d"], "d2h_bytes_per_step": res["d2h"]},
                    "clocks": res["clocks"], "gpu_launches": res["launches"]}
            print(json.dumps(line), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    if args.config == "c5":
        res = run_churn(cfg, args, world, rank, local)
        ms = barrier_max(res["ms"], world)
        kv = barrier_sum(res["kv"], world)
        if rank == 0:
            peak, peak_kind = peaks()
            value = kv / (ms / 1e3) / 1e9
            line = {"metric": "decode attn+append KV-read GB/s", "value": round(value, 2),
                    "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                    "ms_per_step": round(ms / args.steps, 4),
                    "us_per_step": round(1e3 * ms / args.steps, 1),
                    "pct_hbm_peak_per_gpu": round(100 * value / world / peak, 1),
                    "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                    "dtype": "f16 (fp32 accumulate)",
                    "data": "synthetic N(0,1) fp16, seeded churn schedule",
                    "config": dict(base_config, mean_active=round(res["mean_active"], 1),
                                   pool_occupancy=round(res["occupancy"], 3),
                                   pool_blocks=res["pool_blocks"], admitted=res["admitted"],
                                   released=res["released"], preempted=res["preempted"],
                                   prefill_ms_total_timed_apart=round(res["prefill_ms"], 2)),
                    "clocks": res["clocks"], "gpu_launches": res["launches"]}
            print(json.dumps(line), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    res = run_ours(cfg, args, world, rank, local)
    ms = barrier_max(res["ms"], world)
    rank_ms = gather_values(res["ms"], world)
    kv = barrier_sum(res["kv"], world)
    e2e_ms = barrier_max(res["e2e_ms"], world)
    e2e_kv = barrier_sum(res["e2e_kv"], world)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(cfg, args.seed, args.cpu_baseline_seconds)
    if rank == 0:
        value = kv / (ms / 1e3) / 1e9
        achieved = res["dec_bytes"] / (res["dec_ms"] / 1e3) / 1e9
        traffic = None
        tp = ROOT / "profiles" / "dram_traffic.json"
        if tp.exists():
            t = json.loads(tp.read_text()).get(args.config, {}).get(args.layout)
            traffic = t
        line = {"metric": "decode attn+append KV-read GB/s", "value": round(value, 2),
                "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(ms / args.steps, 4),
                "us_per_step": round(1e3 * ms / args.steps, 1),
                "pct_hbm_peak_per_gpu": round(100 * value / world / peak, 1),
                "per_rank_ms_per_step": [round(x / args.steps, 4) for x in rank_ms],
                "higher_is_better": True,
                "scaling": "strong" if args.shard == "head" or world == 1 else args.scaling,
                "vs_baseline": None, "dtype": "f16 (fp32 accumulate)",
                "data": "synthetic N(0,1) fp16 K/V/Q from a seeded generator (no dataset)",
                "config": dict(base_config, global_batch=res["global_b"],
                               seq_len=max(res["lens"])),
                "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                             "unit": "GB/s", "frac": round(achieved / peak, 4),
                             "traffic": traffic, "kernel": "paged_decode_kernel + merge_kernel",
                             "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback"},
                "cpu_baseline": cpu,
                "e2e": {"value": round(e2e_kv / (e2e_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                        "h2d_bytes_per_step": res["h2d"], "d2h_bytes_per_step": res["d2h"]},
                "clocks": res["clocks"], "gpu_launches": res["launches"]}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
