"""Model integration: the reference's Hugging Face hook and a graph-captured decode engine.

* :func:`kernel_attention_forward` / :func:`register` -- drop-in for the
  reference's ``kernel_attention_forward`` (notebook lines 1043-1066): an
  attention function for ``transformers``' ``ALL_ATTENTION_FUNCTIONS`` that
  sends decode steps (one query token) to :func:`ops.decode_attn_gqa` and
  prefill to the library's own SDPA path of ``transformers``.  Like the
  reference it casts q/K/V to fp16 and reads the whole (contiguous) cache
  every step.

* :class:`GraphDecoder` -- greedy decoding for a Llama-architecture
  ``LlamaForCausalLM`` with a preallocated KV cache, fp16 or int8.  Prefill
  runs eagerly (torch SDPA, causal); every decode step -- embeddings, RMSNorm,
  projections, RoPE, the cache append (int8: quantize-on-append of the new
  token only, bit-exact with the reference quantizer), fused decode attention
  over the cache with the sequence length read on the device
  (:func:`ops.decode_attn_gqa_kvcache` / :func:`ops.decode_attn_gqa_int8_kvcache`),
  MLP, LM head and argmax -- is captured once in a CUDA graph and replayed
  per token, so a step costs no Python or launch overhead.  The model's
  weights may be bf16 or fp16; attention runs on the fp16 / int8 cache.  With
  the default rotary embedding the step's attention prologue is two kernels:
  one GEMM against the concatenated q/k/v weights and
  :func:`ops.rope_qkv_append` (RoPE of q and k from tables the model's own
  rotary module filled, q cast to fp16, k/v appended or quantized into the
  cache -- bit-exact with the HF ops it replaces, ``fused_rope=False``).
  With ``fused_model_ops`` (default) the residual adds and RMSNorms are one
  :func:`ops.add_rmsnorm` launch each and the MLP is one GEMM against the
  concatenated gate/up weights plus :func:`ops.silu_mul` and the down GEMM
  (LlamaRMSNorm / SwiGLU arithmetic; only the fp32 sum of squares is
  reduced in a different order); at batch 1 the gate/up projection and the
  SwiGLU are one :func:`ops.gemv_swiglu` launch, and with an fp16 cache the
  q/k/v projection, RoPE and the cache append one :func:`ops.gemv_rope_append`
  launch.

  With ``tp_group`` (a ``torch.distributed`` group, NCCL on GPUs) the decoder
  is tensor-parallel by KV head: each rank keeps the q/k/v projection rows, the
  KV cache and the attention of Hkv/world KV heads (and their query heads),
  and the per-rank attention outputs are all-gathered every layer -- inside
  the captured graph -- before the replicated output projection, MLP and LM
  head, so every rank produces the same tokens.  The gather is NCCL's
  ``all_gather_into_tensor``, or with ``tp_fused=True`` part of the attention
  kernel itself: it stores its output into every rank's receive buffer over
  NVLink and a bounded wait kernel precedes the output projection
  (:mod:`tp_exchange`).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import _native, ops
from . import sharding

HOOK_NAME = "fqkv_decode"

__all__ = ["HOOK_NAME", "kernel_attention_forward", "register", "GraphDecoder"]


def kernel_attention_forward(module, query, key, value, attention_mask=None, scaling=None, dropout=0.0, **kwargs):
    """Attention function for ``ALL_ATTENTION_FUNCTIONS``.

    query [B, Hq, q_len, D], key/value [B, Hkv, kv_len, D] -> ([B, q_len, Hq, D], None).
    Decode (q_len == 1) runs :func:`ops.decode_attn_gqa`; prefill is handed to
    ``transformers``' SDPA attention function, as in the reference.
    """
    q_len = query.shape[2]
    if q_len != 1:
        from transformers.integrations.sdpa_attention import sdpa_attention_forward
        return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout, scaling=scaling,
                                      **kwargs)
    D = query.shape[-1]
    if scaling is not None and not math.isclose(scaling, D ** -0.5, rel_tol=1e-6):
        raise ValueError(f"fqkv decode attention uses scale 1/sqrt(D); got scaling={scaling}")
    q = query[:, :, 0, :].to(torch.float16).contiguous()          # [B, Hq, D]
    K = key.to(torch.float16).contiguous()                          # [B, Hkv, kv, D]
    V = value.to(torch.float16).contiguous()
    out = ops.decode_attn_gqa(q, K, V, 8)                           # [B, Hq, D]
    return out.to(query.dtype).unsqueeze(1), None                   # [B, 1, Hq, D]


def register(name: str = HOOK_NAME) -> str:
    """Register :func:`kernel_attention_forward` under ``name`` in ``ALL_ATTENTION_FUNCTIONS``."""
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    ALL_ATTENTION_FUNCTIONS.register(name, kernel_attention_forward)
    return name


class GraphDecoder:
    """Greedy decode of a ``LlamaForCausalLM`` with a static fp16 KV cache and a CUDA-graph step.

    Usage::

        dec = GraphDecoder(model, batch=B, max_len=P + T)
        first = dec.prefill(prompt_ids)          # [B] first generated token
        tokens = dec.generate(T - 1)             # [B, T - 1] following tokens
    """

    def __init__(self, model, batch: int, max_len: int, keep_logits: bool = False, kv_dtype: str = "fp16",
                 tp_group=None, tp_fused: bool = False, fused_rope: bool = True, fused_model_ops: bool = True):
        from transformers.models.llama.modeling_llama import apply_rotary_pos_emb

        self._rope = apply_rotary_pos_emb
        self.model = model
        cfg = model.config
        self.L = cfg.num_hidden_layers
        self.Hq = cfg.num_attention_heads
        self.Hkv = cfg.num_key_value_heads
        self.D = getattr(cfg, "head_dim", None) or cfg.hidden_size // self.Hq
        self.B = batch
        # tensor parallelism by KV head: this rank's query / KV heads and projection rows
        self.tp_group = tp_group
        if tp_group is not None:
            import torch.distributed as dist
            self.world, self.rank = dist.get_world_size(tp_group), dist.get_rank(tp_group)
        else:
            self.world, self.rank = 1, 0
        sharding.shard_kv_heads(self.Hq, self.Hkv, self.world, self.rank)  # validates divisibility
        self.Hq_l, self.Hkv_l = self.Hq // self.world, self.Hkv // self.world
        self.proj = None
        if self.world > 1:
            self.proj = [sharding.shard_attention_projections(layer.self_attn, self.Hq, self.Hkv, self.D,
                                                              self.world, self.rank)
                         for layer in model.model.layers]
        self.max_len = max_len
        dev = next(model.parameters()).device
        self.dev = dev
        self.dtype = next(model.parameters()).dtype
        if kv_dtype not in ("fp16", "int8"):
            raise ValueError("kv_dtype must be 'fp16' or 'int8'")
        self.kv_dtype = kv_dtype
        cache_dtype = torch.float16 if kv_dtype == "fp16" else torch.int8
        self.kc = torch.zeros(self.L, batch, self.Hkv_l, max_len, self.D, dtype=cache_dtype, device=dev)
        self.vc = torch.zeros_like(self.kc)
        if kv_dtype == "int8":  # per-token fp16 scales of the int8 codes
            self.ks = torch.zeros(self.L, batch, self.Hkv_l, max_len, dtype=torch.float16, device=dev)
            self.vs = torch.zeros_like(self.ks)
        self.pos32 = torch.zeros(1, dtype=torch.int32, device=dev)   # self.pos as int32 (append position)
        self.pos = torch.zeros(1, dtype=torch.long, device=dev)      # position of the token fed to the step
        self.nlen = torch.zeros(1, dtype=torch.int32, device=dev)    # valid cache length during the step
        self.tok = torch.zeros(batch, dtype=torch.long, device=dev)  # token fed to the step
        self.out_tokens = torch.zeros(batch, max_len, dtype=torch.long, device=dev)
        self.attn_out = torch.empty(batch, self.Hq_l, self.D, dtype=torch.float16, device=dev)
        # all-gather staging of the per-rank attention outputs (world x [B, 1, Hq_l, D])
        self.gather_buf = (torch.empty(self.world * batch, 1, self.Hq_l, self.D, dtype=torch.float16, device=dev)
                           if self.world > 1 else None)
        nb = ops.workspace_bytes(kv_dtype, batch, self.Hq_l, self.Hkv_l, max_len, self.D)
        self.ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=dev) if nb else None
        # fused all-gather: receive buffers / counters of every rank mapped here
        self.xchg = None
        if tp_fused and self.world > 1:
            from .tp_exchange import PeerExchange
            self.xchg = PeerExchange(tp_group, self.L, batch, self.Hq_l, self.D, dev)
            fmt = _native.KV_F16 if kv_dtype == "fp16" else _native.KV_INT8
            self.xchg.set_plan(fmt, batch, self.Hq_l, self.Hkv_l, max_len, self.D,
                               self.ws.numel() if self.ws is not None else 0)
        self.keep_logits = keep_logits
        self.logits = torch.zeros(batch, cfg.vocab_size, dtype=torch.float32, device=dev) if keep_logits else None
        # fused attention prologue: concatenated q/k/v weights + rotary tables of every position
        rot = model.model.rotary_emb
        self.rope_fused = (fused_rope and self.dtype in (torch.float16, torch.bfloat16) and self.D in (64, 128)
                           and getattr(rot, "rope_type", "default") == "default"
                           and float(getattr(rot, "attention_scaling", 1.0)) == 1.0)
        if self.rope_fused:
            self.wqkv, self.bqkv = [], []
            for li, layer in enumerate(model.model.layers):
                if self.proj is not None:
                    parts = self.proj[li]
                else:
                    a = layer.self_attn
                    parts = [(lin.weight.detach(), lin.bias.detach() if lin.bias is not None else None)
                             for lin in (a.q_proj, a.k_proj, a.v_proj)]
                self.wqkv.append(torch.cat([w for w, _ in parts], 0).contiguous())
                self.bqkv.append(torch.cat([b for _, b in parts], 0).contiguous() if parts[0][1] is not None else None)
            with torch.no_grad():
                cos, sin = rot(torch.empty(1, 1, 1, dtype=self.dtype, device=dev),
                               torch.arange(max_len, device=dev)[None])
            self.cos_t = cos[0].contiguous()
            self.sin_t = sin[0].contiguous()
            self.q16 = torch.empty(batch, self.Hq_l, self.D, dtype=torch.float16, device=dev)
        # fused residual/RMSNorm and SwiGLU (same dtype conditions, LlamaRMSNorm / silu MLP)
        H = cfg.hidden_size
        self.model_fused = (fused_model_ops and self.rope_fused and H <= 8192
                            and getattr(cfg, "hidden_act", "silu") == "silu"
                            and all(hasattr(l.input_layernorm, "variance_epsilon") for l in model.model.layers))
        if self.model_fused:
            I = cfg.intermediate_size
            self.wgu = [torch.cat([l.mlp.gate_proj.weight.detach(), l.mlp.up_proj.weight.detach()], 0).contiguous()
                        for l in model.model.layers]
            self.bgu = [torch.cat([l.mlp.gate_proj.bias.detach(), l.mlp.up_proj.bias.detach()], 0).contiguous()
                        if l.mlp.gate_proj.bias is not None else None for l in model.model.layers]
            self.xn = torch.empty(batch, H, dtype=self.dtype, device=dev)     # normed hidden state
            self.act = torch.empty(batch, I, dtype=self.dtype, device=dev)   # silu(gate) * up
            # batch <= 4: the q/k/v, o and down projections run on the library's GEMV (measured
            # 1.5-2x faster than cuBLAS's batch-1..4 kernels on B200); gate/up and the LM head stay
            # on cuBLAS, which streams those large matrices near HBM speed.
            self.small_b = batch <= 4 and H % 256 == 0 and I % 256 == 0 and (self.Hq * self.D) % 256 == 0
            if not self.small_b and self.world == 1 and self.dtype == torch.bfloat16:
                # one GPU, batch > 4: attention writes bf16, so cuBLAS's output projection reads it
                # without a cast kernel (each element rounded once from fp32)
                self.attn_out = torch.empty(batch, self.Hq_l, self.D, dtype=torch.bfloat16, device=dev)
            self.arg_scratch = torch.zeros(int(_native.lib().fqkv_argmax_scratch_bytes(batch)), dtype=torch.uint8,
                                           device=dev)
            self.nxt = torch.empty(batch, dtype=torch.long, device=dev)
        self.graph = None
        self.prompt_len = 0

    # ------------------------------------------------------------------ per-rank attention pieces
    def _qkv(self, li: int, attn, x: torch.Tensor):
        """This rank's q [B, Hq_l, T, D], k/v [B, Hkv_l, T, D] projections of x [B, T, H]."""
        B, T = x.shape[0], x.shape[1]
        if self.proj is None:
            q, k, v = attn.q_proj(x), attn.k_proj(x), attn.v_proj(x)
        else:
            (wq, bq), (wk, bk), (wv, bv) = self.proj[li]
            q, k, v = F.linear(x, wq, bq), F.linear(x, wk, bk), F.linear(x, wv, bv)
        return (q.view(B, T, self.Hq_l, self.D).transpose(1, 2), k.view(B, T, self.Hkv_l, self.D).transpose(1, 2),
                v.view(B, T, self.Hkv_l, self.D).transpose(1, 2))

    def _heads(self, o: torch.Tensor, staging=None) -> torch.Tensor:
        """Local attention output o [B, T, Hq_l, D] -> all heads [B, T, Hq*D] (all-gather when sharded)."""
        B, T = o.shape[0], o.shape[1]
        if self.world == 1:
            return o.reshape(B, T, self.Hq * self.D)
        if staging is None:
            staging = torch.empty((self.world * B,) + tuple(o.shape[1:]), dtype=o.dtype, device=o.device)
        return sharding.gather_heads(o.contiguous(), staging, self.world, self.tp_group)

    # ------------------------------------------------------------------ prefill
    @torch.no_grad()
    def prefill(self, ids: torch.Tensor) -> torch.Tensor:
        """Run the prompt [B, P], fill the cache, return the first generated token [B]."""
        m = self.model.model
        B, P = ids.shape
        if B != self.B or P >= self.max_len:
            raise ValueError("prompt does not fit the decoder's batch / max_len")
        h = m.embed_tokens(ids)
        position_ids = torch.arange(P, device=self.dev)[None].expand(B, P)
        cos, sin = m.rotary_emb(h, position_ids=position_ids)
        for li, layer in enumerate(m.layers):
            attn = layer.self_attn
            x = layer.input_layernorm(h)
            q, k, v = self._qkv(li, attn, x)
            q, k = self._rope(q, k, cos, sin)
            self._append(li, k, v, 0)
            o = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
            h = h + attn.o_proj(self._heads(o.transpose(1, 2)))
            h = h + layer.mlp(layer.post_attention_layernorm(h))
        logits = self.model.lm_head(m.norm(h[:, -1:]))[:, -1].float()
        first = logits.argmax(-1)
        self.tok.copy_(first)
        self.pos.fill_(P)
        self.pos32.fill_(P)
        self.nlen.fill_(P + 1)
        self.out_tokens[:, P].copy_(first)
        self.prompt_len = P
        if self.keep_logits:
            self.logits.copy_(logits)
        return first

    # ------------------------------------------------------------------ cache
    def _append(self, li: int, k: torch.Tensor, v: torch.Tensor, pos) -> None:
        """Write k/v [B, Hkv, T, D] at position ``pos`` (int, or the device tensor) of layer li."""
        if self.kv_dtype == "fp16":
            if isinstance(pos, int):
                T = k.shape[2]
                self.kc[li, :, :, pos:pos + T].copy_(k)
                self.vc[li, :, :, pos:pos + T].copy_(v)
            else:
                self.kc[li].index_copy_(2, self.pos, k.to(torch.float16))
                self.vc[li].index_copy_(2, self.pos, v.to(torch.float16))
        else:
            p = pos if isinstance(pos, int) else self.pos32
            ops.quantize_into_cache(k.to(torch.float16).contiguous(), self.kc[li], self.ks[li], p)
            ops.quantize_into_cache(v.to(torch.float16).contiguous(), self.vc[li], self.vs[li], p)

    def _attend(self, li: int, q: torch.Tensor) -> None:
        if self.xchg is not None:  # output goes to every rank's receive buffer of layer li
            ks = self.ks[li] if self.kv_dtype == "int8" else None
            vs = self.vs[li] if self.kv_dtype == "int8" else None
            ops.decode_attn_kvcache_tp(q, self.kc[li], self.vc[li], self.nlen, self.xchg.tp_out[li], ks, vs,
                                       workspace=self.ws)
            return
        if self.kv_dtype == "fp16":
            ops.decode_attn_gqa_kvcache(q, self.kc[li], self.vc[li], self.nlen, out=self.attn_out, workspace=self.ws)
        else:
            ops.decode_attn_gqa_int8_kvcache(q, self.kc[li], self.vc[li], self.ks[li], self.vs[li], self.nlen,
                                             out=self.attn_out, workspace=self.ws)

    # ------------------------------------------------------------------ decode step
    def _step(self) -> None:
        """Decode the token in ``self.tok`` at ``self.pos``; graph-capturable (no host sync)."""
        m = self.model.model
        B = self.B
        if self.model_fused:
            self._step_fused()
            return
        h = m.embed_tokens(self.tok[:, None])                         # [B, 1, H]
        if not self.rope_fused:
            position_ids = self.pos.expand(B)[:, None]
            cos, sin = m.rotary_emb(h, position_ids=position_ids)
        for li, layer in enumerate(m.layers):
            attn = layer.self_attn
            x = layer.input_layernorm(h)
            if self.rope_fused:
                qkv = F.linear(x, self.wqkv[li], self.bqkv[li]).view(B, -1)
                ks = self.ks[li] if self.kv_dtype == "int8" else None
                vs = self.vs[li] if self.kv_dtype == "int8" else None
                ops.rope_qkv_append(qkv, self.cos_t, self.sin_t, self.pos32, self.q16, self.kc[li], self.vc[li],
                                    ks, vs)
                self._attend(li, self.q16)
            else:
                q, k, v = self._qkv(li, attn, x)
                q, k = self._rope(q, k, cos, sin)
                self._append(li, k, v, self.pos)
                self._attend(li, q[:, :, 0].to(torch.float16).contiguous())
            if self.xchg is not None:
                self.xchg.wait()
                o = self.xchg.gathered(li).permute(1, 0, 2, 3).reshape(B, 1, self.Hq * self.D)
            else:
                o = self._heads(self.attn_out.view(B, 1, self.Hq_l, self.D), self.gather_buf)
            h = h + attn.o_proj(o.to(h.dtype))
            h = h + layer.mlp(layer.post_attention_layernorm(h))
        logits = self.model.lm_head(m.norm(h))[:, 0].float()
        nxt = logits.argmax(-1)
        if self.keep_logits:
            self.logits.copy_(logits)
        self.pos.add_(1)
        self.pos32.add_(1)
        self.nlen.add_(1)
        self.out_tokens.index_copy_(1, self.pos, nxt[:, None])
        self.tok.copy_(nxt)

    def _step_fused(self) -> None:
        """The decode step with every launch of the block fused that can be (see the class docstring)."""
        m = self.model.model
        B = self.B
        layers = m.layers
        h = m.embed_tokens(self.tok).view(B, -1)                      # [B, H], residual stream (updated in place)
        x = self.xn
        ops.add_rmsnorm(h, None, layers[0].input_layernorm.weight, x, layers[0].input_layernorm.variance_epsilon)
        for li, layer in enumerate(layers):
            attn = layer.self_attn
            if B == 1 and self.small_b and self.kv_dtype != "int8":
                # q/k/v GEMV with RoPE, the fp16 cast of q and the cache append in its epilogue
                ops.gemv_rope_append(x, self.wqkv[li], self.bqkv[li], self.cos_t, self.sin_t, self.pos32, self.q16,
                                     self.kc[li], self.vc[li])
            else:
                qkv = (ops.gemv(x, self.wqkv[li], self.bqkv[li]) if self.small_b
                       else F.linear(x, self.wqkv[li], self.bqkv[li]))
                ks = self.ks[li] if self.kv_dtype == "int8" else None
                vs = self.vs[li] if self.kv_dtype == "int8" else None
                ops.rope_qkv_append(qkv, self.cos_t, self.sin_t, self.pos32, self.q16, self.kc[li], self.vc[li],
                                    ks, vs)
            self._attend(li, self.q16)
            if self.xchg is not None:
                self.xchg.wait()
                o = self.xchg.gathered(li).permute(1, 0, 2, 3).reshape(B, self.Hq * self.D)
            else:
                o = self._heads(self.attn_out.view(B, 1, self.Hq_l, self.D), self.gather_buf).view(B, -1)
            if self.small_b:
                # the GEMV reads the fp16 attention output and rounds it to the model dtype
                ob = attn.o_proj.bias.detach() if attn.o_proj.bias is not None else None
                a = ops.gemv(o.contiguous(), attn.o_proj.weight.detach(), ob)
            else:
                a = attn.o_proj(o.to(h.dtype))
            ops.add_rmsnorm(h, a, layer.post_attention_layernorm.weight, x,
                            layer.post_attention_layernorm.variance_epsilon)
            if B == 1 and self.small_b:
                # gate/up GEMV with the SwiGLU in its epilogue, one launch (Llama-1B shapes on B200:
                # batch 1 1257 -> 1287 tok/s; batch 4 4023 -> 3660, so larger batches keep cuBLAS)
                ops.gemv_swiglu(x, self.wgu[li], self.bgu[li], out=self.act)
            else:
                gu = F.linear(x, self.wgu[li], self.bgu[li])
                ops.silu_mul(gu, self.act)
            if self.small_b:
                db = layer.mlp.down_proj.bias.detach() if layer.mlp.down_proj.bias is not None else None
                d = ops.gemv(self.act, layer.mlp.down_proj.weight.detach(), db)
            else:
                d = layer.mlp.down_proj(self.act)
            nrm = layers[li + 1].input_layernorm if li + 1 < len(layers) else m.norm
            ops.add_rmsnorm(h, d, nrm.weight, x, nrm.variance_epsilon)
        logits = self.model.lm_head(x)
        nxt = ops.argmax_rows(logits, self.arg_scratch, self.nxt)   # as logits.argmax(-1), multi-CTA
        if self.keep_logits:
            self.logits.copy_(logits)
        self.pos.add_(1)
        self.pos32.add_(1)
        self.nlen.add_(1)
        self.out_tokens.index_copy_(1, self.pos, nxt[:, None])
        self.tok.copy_(nxt)

    @torch.no_grad()
    def capture(self, warmup: int = 2) -> None:
        """Capture one decode step in a CUDA graph (restores the decoder state afterwards)."""
        state = [self.kc, self.vc, self.pos, self.pos32, self.nlen, self.tok, self.out_tokens]
        if self.kv_dtype == "int8":
            state += [self.ks, self.vs]
        if self.keep_logits:
            state.append(self.logits)
        saved = [t.clone() for t in state]
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._step()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()
        for dst, src in zip(state, saved):
            dst.copy_(src)
        torch.cuda.synchronize(self.dev)

    def release(self) -> None:
        """Drop the captured graph (required before destroying a process group whose collectives it holds)
        and, with the fused all-gather, the exchange memory (collective: every rank calls it)."""
        if self.graph is not None:
            self.graph.reset()
            self.graph = None
        if self.xchg is not None:
            self.xchg.close()
            self.xchg = None

    @torch.no_grad()
    def step(self) -> None:
        if self.graph is None:
            self._step()
        else:
            self.graph.replay()

    @torch.no_grad()
    def generate(self, steps: int) -> torch.Tensor:
        """Decode ``steps`` more tokens after :meth:`prefill`; returns them as [B, steps].

        Raises RuntimeError when a bounded wait inside the step's kernels gave up -- with the
        fused tensor-parallel gather, a peer rank that stopped or fell behind (status 64) --
        instead of returning tokens decoded from missing outputs."""
        P = self.prompt_len
        if P + 1 + steps > self.max_len:
            raise ValueError("generation exceeds max_len")
        for _ in range(steps):
            self.step()
        ops.check_device_status(self.dev, "decode step")
        return self.out_tokens[:, P + 1:P + 1 + steps]
