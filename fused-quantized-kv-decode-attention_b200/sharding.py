"""Multi-GPU sharding of decode work: independent units, no data-path collective.

Every (sequence, KV head) unit of decode attention is independent, so a
multi-GPU job splits units across ranks (one process per GPU) and exchanges
nothing but timing.  Two splits are provided:

* by sequence (batch rows) -- each rank owns whole sequences;
* by KV head -- each rank owns Hkv/world KV heads together with the G query
  heads that read them, so no rank ever needs another rank's KV.
"""
from __future__ import annotations

__all__ = ["shard_range", "shard_batch", "shard_kv_heads", "max_over_ranks"]


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [lo, hi) share of `total` units for `rank`; shares differ by at most one."""
    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def shard_batch(B: int, world: int, rank: int) -> slice:
    lo, hi = shard_range(B, world, rank)
    return slice(lo, hi)


def shard_kv_heads(Hq: int, Hkv: int, world: int, rank: int) -> tuple[slice, slice]:
    """(query-head slice, KV-head slice) of `rank`; Hkv must divide evenly across ranks."""
    if Hq % Hkv or Hkv % world:
        raise ValueError(f"Hkv={Hkv} must be a multiple of world={world} and divide Hq={Hq}")
    G = Hq // Hkv
    per = Hkv // world
    return slice(rank * per * G, (rank + 1) * per * G), slice(rank * per, (rank + 1) * per)


def max_over_ranks(value: float, group=None, device=None) -> float:
    """Max of a per-rank float over all ranks (identity without torch.distributed)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
