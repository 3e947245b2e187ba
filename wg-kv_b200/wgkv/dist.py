"""Multi-GPU plumbing for the admission path: one process per GPU.

Nothing on the hot path exchanges data between GPUs: sequences (and KV heads)
are independent in the gate, the compaction, the page tables, the indices and
both attentions.  A job is therefore split into contiguous shards of
sequences (or of KV heads), and each rank owns its own paged pool.  With
sequence sharding the only collective is the timing reduction (max over
ranks); with KV-head sharding the attention output projection around the
path sums its partial products over ranks (``wgkv.tp``).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(n: int, rank: int, world: int):
    """Contiguous [start, end) share of n items for `rank` (earlier ranks take the remainder)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    base, rem = divmod(n, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def kv_head_shard(num_kv_heads: int, num_q_heads: int, rank: int, world: int):
    """KV heads owned by `rank` and the matching query heads (GQA groups stay whole)."""
    h0, h1 = shard_range(num_kv_heads, rank, world)
    g = num_q_heads // num_kv_heads
    return (h0, h1), (h0 * g, h1 * g)


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank scalar (e.g. a CUDA-event time) over the process group; identity when alone."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, device=None) -> float:
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())
