"""float64 restatement of the reference's single-query decode attention.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

What the reference computes (every kernel in ``kernels/*.cu``):

* per query row r: ``s_i = (q . K_i) * (1/sqrt(D))`` in fp32
  (``kernels/decode_attn_fp16_mw.cu:22-25``), ``o = softmax(s) . V`` with an
  online max / denominator (``:26-30``) merged across warps (``:32-48``),
  output rounded once to fp16 (``:47``);
* quantized KV is dequantised in registers as ``code * scale``
  (``kernels/decode_attn_int8_mw.cu:24,31``, ``kernels/decode_attn_int4.cu:21-31``);
* GQA: query head h of batch b reads KV head ``h // G`` with ``G = Hq // Hkv``
  (``kernels/decode_attn_gqa.cu:13,16-17``);
* split-K: split ``s`` covers keys ``[s*chunk, min(N, (s+1)*chunk))`` with
  ``chunk = ceil(N/S)`` (``kernels/decode_attn_gqa_sk_fast.cu:13``) and emits
  an unnormalised fp32 partial ``(m, l, o)`` (``:49-52``); the combine merges
  partials with log-sum-exp weights, treating an empty split (``m = -inf``)
  as weight 0 (``:66-73``, ``:80-93``).

The oracle evaluates the exact softmax in float64 (the fp32-accumulated
reference is within ~1e-6 of it), which is the quantity the GPU kernels are
compared against with ``atol=2e-3, rtol=1e-2``.
"""
from __future__ import annotations

import math

import numpy as np

__all__ = [
    "decode_attention",
    "decode_attention_gqa",
    "splitk_partials",
    "splitk_combine",
    "sdpa_cpu_reference_path",
]


def decode_attention(q: np.ndarray, K: np.ndarray, V: np.ndarray,
                     scale: float | None = None) -> np.ndarray:
    """q [R, D], K/V [R, N, D] (any float dtype) -> o [R, D] float64."""
    q = np.asarray(q, np.float64)
    K = np.asarray(K, np.float64)
    V = np.asarray(V, np.float64)
    D = q.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    s = np.einsum("rnd,rd->rn", K, q) * scale
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("rn,rnd->rd", p, V)


def decode_attention_gqa(q: np.ndarray, K: np.ndarray, V: np.ndarray) -> np.ndarray:
    """q [B, Hq, D], K/V [B, Hkv, N, D] -> o [B, Hq, D] float64 (KV head h // G)."""
    q = np.asarray(q, np.float64)
    B, Hq, D = q.shape
    Hkv = K.shape[1]
    G = Hq // Hkv
    Ke = np.repeat(np.asarray(K, np.float64), G, axis=1)   # repeat_interleave
    Ve = np.repeat(np.asarray(V, np.float64), G, axis=1)
    N = Ke.shape[2]
    o = decode_attention(q.reshape(B * Hq, D), Ke.reshape(B * Hq, N, D),
                         Ve.reshape(B * Hq, N, D))
    return o.reshape(B, Hq, D)


def splitk_partials(q: np.ndarray, K: np.ndarray, V: np.ndarray, S: int):
    """Per-split ``(m, l, o)`` of the reference partial kernel (natural-log m).

    q [Hq, D], K/V [Hkv, N, D] -> m [Hq, S], l [Hq, S], o [Hq, S, D] float64;
    empty splits carry ``m = -inf, l = 0, o = 0``.
    """
    q = np.asarray(q, np.float64)
    K = np.asarray(K, np.float64)
    V = np.asarray(V, np.float64)
    Hq, D = q.shape
    Hkv, N, _ = K.shape
    G = Hq // Hkv
    chunk = (N + S - 1) // S
    scale = 1.0 / math.sqrt(D)
    m = np.full((Hq, S), -np.inf)
    l = np.zeros((Hq, S))
    o = np.zeros((Hq, S, D))
    for h in range(Hq):
        kv = h // G
        for s in range(S):
            lo, hi = s * chunk, min(N, (s + 1) * chunk)
            if lo >= hi:
                continue
            sc = K[kv, lo:hi] @ q[h] * scale
            m[h, s] = sc.max()
            p = np.exp(sc - m[h, s])
            l[h, s] = p.sum()
            o[h, s] = p @ V[kv, lo:hi]
    return m, l, o


def splitk_combine(m: np.ndarray, l: np.ndarray, o: np.ndarray) -> np.ndarray:
    """Log-sum-exp merge of split partials; ``m = -inf`` splits get weight 0."""
    M = m.max(axis=-1, keepdims=True)
    with np.errstate(invalid="ignore"):
        w = np.where(np.isneginf(m), 0.0, np.exp(m - M))
    L = (w * l).sum(axis=-1)
    return (w[..., None] * o).sum(axis=-2) / L[..., None]


def sdpa_cpu_reference_path(q, K, V):
    """The reference's own CPU attention path (``tests/test_kernels.py:14-16``).

    ``F.scaled_dot_product_attention`` on CPU fp16 tensors, q [R, D], K/V
    [R, N, D] (torch tensors) -> o [R, D] fp16.  Used as the timed CPU
    baseline; imported lazily so the numpy oracle needs no torch.
    """
    import torch.nn.functional as F
    R, D = q.shape
    N = K.shape[1]
    return F.scaled_dot_product_attention(
        q.view(R, 1, 1, D), K.view(R, 1, N, D), V.view(R, 1, N, D)).view(R, D)
