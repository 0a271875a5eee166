"""Multi-rank logic on CPU (gloo, world_size 2): shards cover every unit once,
KV-head shards keep each query head with its KV head, and the max-over-ranks
timing reduction returns the slowest rank.  No GPU is used."""
from __future__ import annotations

import os

import pytest
import torch.multiprocessing as mp

from conftest import load_package


def _worker(rank: int, world: int, port: int, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = load_package().sharding
        mine = list(range(*sh.shard_range(64, world, rank)))
        got = [None] * world
        dist.all_gather_object(got, mine)
        qs, ks = sh.shard_kv_heads(32, 8, world, rank)
        heads = [None] * world
        dist.all_gather_object(heads, (qs.start, qs.stop, ks.start, ks.stop))
        m = sh.max_over_ranks(1.0 + rank * 2.5)
        q.put((rank, got, heads, m))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharding_and_max_reduction():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, got, heads, m in results:
        flat = sorted(u for part in got for u in part)
        assert flat == list(range(64))                       # every sequence exactly once
        for qs0, qs1, ks0, ks1 in heads:                      # query heads follow their KV heads
            assert (qs1 - qs0) == 4 * (ks1 - ks0)
            assert all(h // 4 in range(ks0, ks1) for h in range(qs0, qs1))
        assert m == pytest.approx(3.5)                       # slowest rank wins


def test_shard_range_balanced():
    sh = load_package().sharding
    for total in (0, 1, 7, 64, 1000):
        for world in (1, 2, 3, 8):
            spans = [sh.shard_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [h - l for l, h in spans]
            assert max(sizes) - min(sizes) <= 1


def _tp_worker(rank: int, world: int, port: int, q):
    """Tensor-parallel attention block on CPU (gloo): sharded q/k/v rows, local GQA
    attention, all-gather into head order, replicated o_proj -- against the
    unsharded block on the same weights."""
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaAttention

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = load_package().sharding
        torch.manual_seed(0)
        Hq, Hkv, D, H = 8, 4, 16, 64
        cfg = LlamaConfig(hidden_size=H, num_attention_heads=Hq, num_key_value_heads=Hkv, head_dim=D,
                          attention_bias=True)
        attn = LlamaAttention(cfg, layer_idx=0).float()
        for p in attn.parameters():
            torch.nn.init.normal_(p, std=0.2)
        B, T = 3, 5
        x = torch.randn(B, T, H)

        def block(qp, kp, vp, hq, hkv):
            qq = F.linear(x, *qp).view(B, T, hq, D).transpose(1, 2)
            kk = F.linear(x, *kp).view(B, T, hkv, D).transpose(1, 2)
            vv = F.linear(x, *vp).view(B, T, hkv, D).transpose(1, 2)
            return F.scaled_dot_product_attention(qq, kk, vv, is_causal=True, enable_gqa=True).transpose(1, 2)

        full = block((attn.q_proj.weight, attn.q_proj.bias), (attn.k_proj.weight, attn.k_proj.bias),
                     (attn.v_proj.weight, attn.v_proj.bias), Hq, Hkv)
        ref = attn.o_proj(full.reshape(B, T, Hq * D))
        qp, kp, vp = sh.shard_attention_projections(attn, Hq, Hkv, D, world, rank)
        local = block(qp, kp, vp, Hq // world, Hkv // world).contiguous()
        staging = torch.empty((world * B,) + tuple(local.shape[1:]))
        out = attn.o_proj(sh.gather_heads(local, staging, world))
        q.put((rank, float((out - ref).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tensor_parallel_attention_block_matches_unsharded(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + world + (os.getpid() % 500)
    procs = [ctx.Process(target=_tp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err in results:
        assert err < 1e-5, (rank, err)
