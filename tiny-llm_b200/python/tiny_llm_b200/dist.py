"""Multi-GPU layer of the paged decode path: one process per GPU.

Two ways to split the work across the GPUs of one node:

* batch shard — each rank owns whole sequences (its own pool, block tables
  and stream); ranks never exchange data on the decode path.
* head shard — for long-context GQA (few sequences, many tokens), rank r
  owns KV heads [r*Hkv/N, (r+1)*Hkv/N) of every sequence and the Hq/N query
  heads that read them; after each layer's decode the per-rank output slices
  are all-gathered so every rank holds all heads, in rank-major layout
  [N][B][Hq/N][D] (the consumer indexes it that way; no transpose).

The collectives here go through torch.distributed (NCCL on GPUs, gloo on
CPU for the tests); the paged kernels themselves are in libtllm_kv.so.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class HeadSlice:
    kv_first: int
    kv_count: int
    q_first: int
    q_count: int


def head_shard(num_kv_heads: int, num_q_heads: int, world: int, rank: int) -> HeadSlice:
    """KV and query heads owned by `rank` when heads are split over `world` GPUs."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV heads do not split over {world} GPUs")
    if num_q_heads % num_kv_heads:
        raise ValueError("num_q_heads must be a multiple of num_kv_heads")
    kv = num_kv_heads // world
    g = num_q_heads // num_kv_heads
    return HeadSlice(rank * kv, kv, rank * kv * g, kv * g)


def batch_shard(lengths: list[int], world: int) -> list[list[int]]:
    """Sequence indices per rank, balancing the KV bytes (sum of lengths):
    longest first onto the least-loaded rank; ties go to the lower rank."""
    if world <= 0:
        raise ValueError("world must be positive")
    load = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda j: (-lengths[j], j)):
        r = min(range(world), key=lambda k: (load[k], k))
        out[r].append(i)
        load[r] += lengths[i]
    return [sorted(x) for x in out]


def _tensor(value: float, group):
    import torch
    import torch.distributed as dist
    backend = dist.get_backend(group)
    dev = "cuda" if backend == "nccl" else "cpu"
    return torch.tensor([float(value)], dtype=torch.float64, device=dev)


def reduce_max(value: float, group=None) -> float:
    """Max of a host scalar over the ranks (e.g. per-rank step time)."""
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    t = _tensor(value, group)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def reduce_sum(value: float, group=None) -> float:
    import torch.distributed as dist
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    t = _tensor(value, group)
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return float(t.item())


def gather_head_outputs(local_out, gathered, group=None) -> None:
    """All-gathers each rank's decode output slice [B][Hq/N][D] into
    `gathered` [N][B][Hq/N][D] (rank-major), in stream order on the current
    stream (NCCL) or synchronously (gloo)."""
    import torch.distributed as dist
    local = local_out.contiguous()
    # concatenated form [N*B][Hq/N][D]: accepted by both NCCL and gloo
    dist.all_gather_into_tensor(gathered.view(-1, *local.shape[1:]), local, group=group)


def connect_peer_gather(cache, gather_bytes: int, group=None) -> None:
    """Sets up the NVLink peer gather of a head-sharded cache: allocates this
    rank's gather region, exchanges the CUDA IPC handles over the process
    group (host objects only) and opens every peer's region."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    mine = cache.peer_init(rank, world, gather_bytes)
    handles = [None] * world
    dist.all_gather_object(handles, mine, group=group)
    cache.peer_connect(handles)


def rank_major_to_heads(gathered):
    """[N][B][Hq/N][D] -> [B][Hq][D] (reference-order view; copies)."""
    n, b, hq_local, d = gathered.shape
    return gathered.permute(1, 0, 2, 3).reshape(b, n * hq_local, d)
