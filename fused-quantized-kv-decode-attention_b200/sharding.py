"""Multi-GPU sharding of decode work: independent units, no data-path collective.

Every (sequence, KV head) unit of decode attention is independent, so a
multi-GPU job splits units across ranks (one process per GPU) and exchanges
nothing but timing.  Two splits are provided:

* by sequence (batch rows) -- each rank owns whole sequences;
* by KV head -- each rank owns Hkv/world KV heads together with the G query
  heads that read them, so no rank ever needs another rank's KV.

Tensor-parallel model decode (config 5 on several GPUs) uses the KV-head
split: :func:`shard_attention_projections` cuts a Llama attention block's
q/k/v projections by output rows, each rank attends over its own heads, and
:func:`gather_heads` all-gathers the per-rank attention outputs (NCCL over
NVLink on GPUs) back into head order for the replicated output projection.
"""
from __future__ import annotations

__all__ = ["shard_range", "shard_batch", "shard_kv_heads", "shard_attention_projections", "gather_heads",
           "max_over_ranks"]


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


def shard_attention_projections(attn, Hq: int, Hkv: int, D: int, world: int, rank: int):
    """Row shards of ``attn.q_proj/k_proj/v_proj`` for ``rank``: ((Wq, bq), (Wk, bk), (Wv, bv)).

    Rank r keeps query heads [r*Hq/world, (r+1)*Hq/world) and the KV heads they
    read, [r*Hkv/world, (r+1)*Hkv/world): local query head i reads local KV head
    i // (Hq/Hkv), exactly as in the unsharded model.  Weights are copied
    (contiguous); biases are None when the projection has none.
    """
    qs, ks = shard_kv_heads(Hq, Hkv, world, rank)

    def rows(lin, sl):
        w = lin.weight.detach()[sl.start * D:sl.stop * D].contiguous()
        b = lin.bias.detach()[sl.start * D:sl.stop * D].contiguous() if lin.bias is not None else None
        return w, b
    return rows(attn.q_proj, qs), rows(attn.k_proj, ks), rows(attn.v_proj, ks)


def gather_heads(local, staging, world: int, group=None):
    """All-gather per-rank attention outputs into head order.

    local [B, T, Hl, D] (contiguous) on every rank -> [B, T, world*Hl*D], the
    heads of rank 0 first.  ``staging`` is a [world*B, T, Hl, D] buffer of the
    same dtype (preallocated, so a CUDA graph can hold the collective).
    """
    import torch.distributed as dist

    dist.all_gather_into_tensor(staging, local, group=group)
    B, T = local.shape[0], local.shape[1]
    return staging.view(world, B, T, *local.shape[2:]).permute(1, 2, 0, 3, 4).reshape(B, T, -1)


def max_over_ranks(value: float, group=None, device=None) -> float:
    """Max of a per-rank float over all ranks (identity without torch.distributed)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
