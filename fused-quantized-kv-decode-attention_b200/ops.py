"""PyTorch-facing operators: the reference extension's surface, on libfqkv_b200.

Each function keeps the name, argument order, output and error behaviour of
the reference operator it replaces (a ``RuntimeError`` whose message starts
with the reference's ``TORCH_CHECK`` keyword: ``cuda``, ``fp16``, ``contig``,
``D``, ``W``, ``CW``, ``int8``, ``packed uint8``, ``launch``), so
``m.decode_attn_fp16_mw(q, K, V, W)`` call sites work unchanged.  The checks
are a superset of the reference's (device, dtype, contiguity and shape are
checked on every tensor of every op).

Work is launched on the current torch CUDA stream of the input's device.
There is no CPU path: inputs must be CUDA tensors and the native library must
be built.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native

__all__ = [
    "decode_attn_fp16_mw",
    "decode_attn_int8_mw",
    "decode_attn_int4",
    "decode_attn_gqa",
    "decode_attn_gqa_kvcache",
    "decode_attn_gqa_int8",
    "decode_attn_gqa_int8_kvcache",
    "quantize_into_cache",
    "gqa_sk_fast",
    "qpt",
    "quant_int4_per_token",
    "workspace_bytes",
]


def _fail(op: str, key: str, detail: str) -> None:
    raise RuntimeError(f"{key}: {op}: {detail}")


def _require_cuda(op: str, *ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            _fail(op, "cuda", "all tensors must be CUDA tensors (there is no CPU path)")
        if t.device != dev:
            _fail(op, "cuda", "all tensors must be on the same device")
    return dev


def _require_dtype(op: str, key: str, dtype: torch.dtype, **ts: torch.Tensor) -> None:
    for name, t in ts.items():
        if t.dtype != dtype:
            _fail(op, key, f"{name} must be {dtype} (got {t.dtype})")


def _require_contig(op: str, **ts: torch.Tensor) -> None:
    for name, t in ts.items():
        if not t.is_contiguous():
            _fail(op, "contig", f"{name} must be contiguous")


def _require_shape(op: str, name: str, t: torch.Tensor, shape: tuple) -> None:
    if tuple(t.shape) != tuple(shape):
        _fail(op, "shape", f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")


def _require_W(op: str, W: int) -> None:
    if int(W) not in (2, 4, 8):
        _fail(op, "W", f"W must be 2, 4 or 8 (got {W})")


def _require_D(op: str, D: int) -> None:
    if D not in (64, 128):
        _fail(op, "D", f"head_dim must be 64 or 128 (got {D})")


class _DeviceGuard:
    """Make `dev` the current CUDA device for the C ABI call (cheap when it already is)."""

    __slots__ = ("dev", "prev")

    def __init__(self, dev: torch.device):
        self.dev = dev.index if dev.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.dev:
            self.prev = cur
            torch.cuda.set_device(self.dev)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def workspace_bytes(kv_format: str, B: int, Hq: int, Hkv: int, N: int, D: int) -> int:
    """Split-K workspace the library would like for this shape on the current device."""
    fmt = {"fp16": _native.KV_F16, "int8": _native.KV_INT8, "int4": _native.KV_INT4}[kv_format]
    return int(_native.lib().fqkv_decode_workspace_bytes(fmt, B, Hq, Hkv, N, D))


def _workspace(fmt: int, dev: torch.device, B: int, Hq: int, Hkv: int, N: int, D: int):
    nbytes = int(_native.lib().fqkv_decode_workspace_bytes(fmt, B, Hq, Hkv, N, D))
    if nbytes == 0:
        return None, 0
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    return ws, nbytes


def decode_attn_fp16_mw(q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, W: int) -> torch.Tensor:
    """fp16 single-query decode: q [R,D], K/V [R,N,D] -> o [R,D] (fp32 accumulation).

    Replaces ``decode_attn_fp16_mw`` (kernels/decode_attn_fp16_mw.cu:50-63).
    """
    op = "decode_attn_fp16_mw"
    dev = _require_cuda(op, q, K, V)
    _require_dtype(op, "fp16", torch.float16, q=q, K=K, V=V)
    _require_contig(op, q=q, K=K, V=V)
    if K.dim() != 3:
        _fail(op, "shape", "K must be [R, N, D]")
    R, N, D = K.shape
    _require_D(op, D)
    _require_W(op, W)
    _require_shape(op, "V", V, (R, N, D))
    _require_shape(op, "q", q, (R, D))
    o = torch.empty((R, D), dtype=torch.float16, device=dev)
    with _DeviceGuard(dev):
        ws, nb = _workspace(_native.KV_F16, dev, R, 1, 1, N, D) if R and N else (None, 0)
        rc = _native.lib().fqkv_decode_attn_fp16_mw(
            q.data_ptr(), K.data_ptr(), V.data_ptr(), o.data_ptr(), R, N, D, int(W),
            ws.data_ptr() if ws is not None else None, nb, _stream(dev))
    _native.check(rc, f"launch: {op}")
    return o


def _quant_decode(op: str, fmt: int, q, K, V, Ks, Vs, W, code_dtype, key, D_of_K):
    dev = _require_cuda(op, q, K, V, Ks, Vs)
    _require_dtype(op, key, code_dtype, K=K, V=V)
    _require_dtype(op, "fp16", torch.float16, q=q, Ks=Ks, Vs=Vs)
    _require_contig(op, q=q, K=K, V=V, Ks=Ks, Vs=Vs)
    if K.dim() != 3:
        _fail(op, "shape", "K must be [R, N, row_bytes]")
    R, N, H = K.shape
    D = D_of_K(H)
    _require_D(op, D)
    _require_W(op, W)
    _require_shape(op, "V", V, (R, N, H))
    _require_shape(op, "Ks", Ks, (R, N))
    _require_shape(op, "Vs", Vs, (R, N))
    _require_shape(op, "q", q, (R, D))
    o = torch.empty((R, D), dtype=torch.float16, device=dev)
    fn = _native.lib().fqkv_decode_attn_int8_mw if fmt == _native.KV_INT8 else _native.lib().fqkv_decode_attn_int4
    with _DeviceGuard(dev):
        ws, nb = _workspace(fmt, dev, R, 1, 1, N, D) if R and N else (None, 0)
        rc = fn(q.data_ptr(), K.data_ptr(), V.data_ptr(), Ks.data_ptr(), Vs.data_ptr(), o.data_ptr(),
                R, N, D, int(W), ws.data_ptr() if ws is not None else None, nb, _stream(dev))
    _native.check(rc, f"launch: {op}")
    return o


def decode_attn_int8_mw(q, K, V, Ks, Vs, W):
    """int8-KV decode: q [R,D] f16, K/V [R,N,D] int8, Ks/Vs [R,N] f16 -> o [R,D] f16.

    Replaces ``decode_attn_int8_mw`` (kernels/decode_attn_int8_mw.cu:52-64).
    """
    return _quant_decode("decode_attn_int8_mw", _native.KV_INT8, q, K, V, Ks, Vs, W, torch.int8, "int8",
                         lambda H: H)


def decode_attn_int4(q, K, V, Ks, Vs, W):
    """int4-KV decode: q [R,D] f16, K/V [R,N,D/2] uint8 (packed), Ks/Vs [R,N] f16 -> o [R,D].

    Replaces ``decode_attn_int4`` (kernels/decode_attn_int4.cu:47-57); D may be
    64 or 128 (the reference accepts only 64).
    """
    return _quant_decode("decode_attn_int4", _native.KV_INT4, q, K, V, Ks, Vs, W, torch.uint8,
                         "packed uint8", lambda H: 2 * H)


def decode_attn_gqa(q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, W: int) -> torch.Tensor:
    """GQA decode: q [B,Hq,D], K/V [B,Hkv,N,D] -> o [B,Hq,D]; head h reads KV head h // (Hq/Hkv).

    Replaces ``decode_attn_gqa`` (kernels/decode_attn_gqa.cu:56-68).  Each KV
    head is read once for all of its query heads.
    """
    op = "decode_attn_gqa"
    dev = _require_cuda(op, q, K, V)
    _require_dtype(op, "fp16", torch.float16, q=q, K=K, V=V)
    _require_contig(op, q=q, K=K, V=V)
    if q.dim() != 3 or K.dim() != 4:
        _fail(op, "shape", "q must be [B, Hq, D] and K [B, Hkv, N, D]")
    B, Hq, D = q.shape
    _, Hkv, N, _ = K.shape
    _require_D(op, D)
    _require_W(op, W)
    _require_shape(op, "K", K, (B, Hkv, N, D))
    _require_shape(op, "V", V, (B, Hkv, N, D))
    if Hkv < 1 or Hq % Hkv:
        _fail(op, "shape", f"Hq ({Hq}) must be a multiple of Hkv ({Hkv})")
    o = torch.empty((B, Hq, D), dtype=torch.float16, device=dev)
    with _DeviceGuard(dev):
        ws, nb = _workspace(_native.KV_F16, dev, B, Hq, Hkv, N, D) if B and N else (None, 0)
        rc = _native.lib().fqkv_decode_attn_gqa(
            q.data_ptr(), K.data_ptr(), V.data_ptr(), o.data_ptr(), B, Hq, Hkv, N, D, int(W),
            ws.data_ptr() if ws is not None else None, nb, _stream(dev))
    _native.check(rc, f"launch: {op}")
    return o


def _kv_out(op: str, q: torch.Tensor, out, shape, dev) -> torch.Tensor:
    """Output of a KV-cache decode call: a new fp16 tensor, or the caller's fp16 / bf16 one."""
    if out is None:
        return torch.empty(shape, dtype=torch.float16, device=dev)
    _require_cuda(op, q, out)
    if out.dtype not in (torch.float16, torch.bfloat16):
        _fail(op, "dtype", f"out must be fp16 or bf16 (got {out.dtype})")
    _require_contig(op, out=out)
    _require_shape(op, "out", out, shape)
    return out


def decode_attn_gqa_kvcache(q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, seq_len,
                            out: torch.Tensor | None = None,
                            workspace: torch.Tensor | None = None) -> torch.Tensor:
    """GQA decode over a preallocated fp16 KV cache (one model decode step).

    q [B,Hq,D] f16; K/V [B,Hkv,max_len,D] f16 with positions [0, n) valid.
    ``seq_len`` is an int (n) or a CUDA int32 tensor holding n, read on the
    device -- with ``out`` and ``workspace`` preallocated the call allocates
    nothing and can be captured in a CUDA graph that is replayed as the cache
    grows.  ``workspace`` needs ``workspace_bytes("fp16", B, Hq, Hkv, max_len, D)``
    bytes (device length) or the same with N = n (host length); too small
    only reduces the split count.  ``out`` may be bf16 (a bf16 model's output
    projection reads it without a cast; each element is rounded once).
    """
    op = "decode_attn_gqa_kvcache"
    dev = _require_cuda(op, q, K, V)
    _require_dtype(op, "fp16", torch.float16, q=q, K=K, V=V)
    _require_contig(op, q=q, K=K, V=V)
    if q.dim() != 3 or K.dim() != 4:
        _fail(op, "shape", "q must be [B, Hq, D] and K [B, Hkv, max_len, D]")
    B, Hq, D = q.shape
    _, Hkv, max_len, _ = K.shape
    _require_D(op, D)
    _require_shape(op, "K", K, (B, Hkv, max_len, D))
    _require_shape(op, "V", V, (B, Hkv, max_len, D))
    if Hkv < 1 or Hq % Hkv:
        _fail(op, "shape", f"Hq ({Hq}) must be a multiple of Hkv ({Hkv})")
    if isinstance(seq_len, torch.Tensor):
        if seq_len.device != dev or seq_len.dtype != torch.int32 or seq_len.numel() < 1:
            _fail(op, "seq_len", "a tensor seq_len must be a CUDA int32 tensor on the inputs' device")
        n_host, n_ptr, n_plan = 0, seq_len.data_ptr(), max_len
    else:
        n_host, n_ptr, n_plan = int(seq_len), None, int(seq_len)
    out = _kv_out(op, q, out, (B, Hq, D), dev)
    with _DeviceGuard(dev):
        if workspace is None:
            ws, nb = _workspace(_native.KV_F16, dev, B, Hq, Hkv, max(n_plan, 1), D) if B else (None, 0)
        else:
            ws, nb = workspace, workspace.numel() * workspace.element_size()
        if out.dtype == torch.bfloat16:
            rc = _native.lib().fqkv_decode_attn_kvcache_out(
                _native.KV_F16, 1, q.data_ptr(), K.data_ptr(), V.data_ptr(), None, None, out.data_ptr(), B, Hq, Hkv,
                max_len, D, n_host, n_ptr, ws.data_ptr() if ws is not None and nb else None, nb, _stream(dev))
            _native.check(rc, f"launch: {op}")
            return out
        rc = _native.lib().fqkv_decode_attn_gqa_kvcache(
            q.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr(), B, Hq, Hkv, max_len, D, n_host, n_ptr,
            ws.data_ptr() if ws is not None and nb else None, nb, _stream(dev))
    _native.check(rc, f"launch: {op}")
    return out


def _seq_len_args(op, seq_len, dev, max_len):
    if isinstance(seq_len, torch.Tensor):
        if seq_len.device != dev or seq_len.dtype != torch.int32 or seq_len.numel() < 1:
            _fail(op, "seq_len", "a tensor seq_len must be a CUDA int32 tensor on the inputs' device")
        return 0, seq_len.data_ptr(), max_len
    return int(seq_len), None, int(seq_len)


def _check_int8_gqa(op, q, Kq, Vq, Ks, Vs):
    dev = _require_cuda(op, q, Kq, Vq, Ks, Vs)
    _require_dtype(op, "int8", torch.int8, Kq=Kq, Vq=Vq)
    _require_dtype(op, "fp16", torch.float16, q=q, Ks=Ks, Vs=Vs)
    _require_contig(op, q=q, Kq=Kq, Vq=Vq, Ks=Ks, Vs=Vs)
    if q.dim() != 3 or Kq.dim() != 4:
        _fail(op, "shape", "q must be [B, Hq, D] and Kq [B, Hkv, N, D]")
    B, Hq, D = q.shape
    _, Hkv, N, _ = Kq.shape
    _require_D(op, D)
    _require_shape(op, "Kq", Kq, (B, Hkv, N, D))
    _require_shape(op, "Vq", Vq, (B, Hkv, N, D))
    _require_shape(op, "Ks", Ks, (B, Hkv, N))
    _require_shape(op, "Vs", Vs, (B, Hkv, N))
    if Hkv < 1 or Hq % Hkv:
        _fail(op, "shape", f"Hq ({Hq}) must be a multiple of Hkv ({Hkv})")
    return dev, B, Hq, Hkv, N, D


def decode_attn_gqa_int8(q, Kq, Vq, Ks, Vs) -> torch.Tensor:
    """GQA decode over int8 KV: q [B,Hq,D] f16, Kq/Vq [B,Hkv,N,D] int8, Ks/Vs [B,Hkv,N] f16 -> [B,Hq,D].

    int8 codes and scales as produced by :func:`qpt`; KV head h // (Hq/Hkv).
    """
    op = "decode_attn_gqa_int8"
    dev, B, Hq, Hkv, N, D = _check_int8_gqa(op, q, Kq, Vq, Ks, Vs)
    o = torch.empty((B, Hq, D), dtype=torch.float16, device=dev)
    with _DeviceGuard(dev):
        ws, nb = _workspace(_native.KV_INT8, dev, B, Hq, Hkv, N, D) if B and N else (None, 0)
        rc = _native.lib().fqkv_decode_attn_gqa_int8(
            q.data_ptr(), Kq.data_ptr(), Vq.data_ptr(), Ks.data_ptr(), Vs.data_ptr(), o.data_ptr(),
            B, Hq, Hkv, N, D, ws.data_ptr() if ws is not None else None, nb, _stream(dev))
    _native.check(rc, f"launch: {op}")
    return o


def decode_attn_gqa_int8_kvcache(q, Kq, Vq, Ks, Vs, seq_len, out=None, workspace=None) -> torch.Tensor:
    """GQA decode over a preallocated int8 KV cache (codes [B,Hkv,max_len,D], scales [B,Hkv,max_len]).

    ``seq_len``, ``out`` and ``workspace`` as in :func:`decode_attn_gqa_kvcache`.
    """
    op = "decode_attn_gqa_int8_kvcache"
    dev, B, Hq, Hkv, max_len, D = _check_int8_gqa(op, q, Kq, Vq, Ks, Vs)
    n_host, n_ptr, n_plan = _seq_len_args(op, seq_len, dev, max_len)
    out = _kv_out(op, q, out, (B, Hq, D), dev)
    with _DeviceGuard(dev):
        if workspace is None:
            ws, nb = _workspace(_native.KV_INT8, dev, B, Hq, Hkv, max(n_plan, 1), D) if B else (None, 0)
        else:
            ws, nb = workspace, workspace.numel() * workspace.element_size()
        if out.dtype == torch.bfloat16:
            rc = _native.lib().fqkv_decode_attn_kvcache_out(
                _native.KV_INT8, 1, q.data_ptr(), Kq.data_ptr(), Vq.data_ptr(), Ks.data_ptr(), Vs.data_ptr(),
                out.data_ptr(), B, Hq, Hkv, max_len, D, n_host, n_ptr,
                ws.data_ptr() if ws is not None and nb else None, nb, _stream(dev))
            _native.check(rc, f"launch: {op}")
            return out
        rc = _native.lib().fqkv_decode_attn_gqa_int8_kvcache(
            q.data_ptr(), Kq.data_ptr(), Vq.data_ptr(), Ks.data_ptr(), Vs.data_ptr(), out.data_ptr(),
            B, Hq, Hkv, max_len, D, n_host, n_ptr, ws.data_ptr() if ws is not None and nb else None, nb,
            _stream(dev))
    _native.check(rc, f"launch: {op}")
    return out


def quantize_into_cache(X: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor, pos, int4: bool = False) -> None:
    """Quantize-on-append: X [..., T, D] f16 -> codes[..., pos:pos+T, :], scales[..., pos:pos+T] of a cache.

    codes [..., cap, D] int8 (int4: [..., cap, D/2] uint8), scales [..., cap] f16;
    bit-exact with :func:`qpt` / :func:`quant_int4_per_token`.  ``pos`` is an
    int or a CUDA int32 tensor read on the device (graph-capturable append).
    """
    op = "quantize_into_cache"
    dev = _require_cuda(op, X, codes, scales)
    _require_dtype(op, "fp16", torch.float16, X=X, scales=scales)
    _require_dtype(op, "packed uint8" if int4 else "int8", torch.uint8 if int4 else torch.int8, codes=codes)
    _require_contig(op, X=X, codes=codes, scales=scales)
    if X.dim() < 2 or codes.dim() != X.dim() or scales.dim() != X.dim() - 1:
        _fail(op, "shape", "X [..., T, D], codes [..., cap, D or D/2], scales [..., cap]")
    D, T, cap = X.shape[-1], X.shape[-2], codes.shape[-2]
    G = X.numel() // (T * D) if T and D else 0
    _require_D(op, D)
    _require_shape(op, "codes", codes, tuple(X.shape[:-2]) + (cap, D // 2 if int4 else D))
    _require_shape(op, "scales", scales, tuple(X.shape[:-2]) + (cap,))
    if isinstance(pos, torch.Tensor):
        if pos.device != dev or pos.dtype != torch.int32:
            _fail(op, "pos", "a tensor pos must be a CUDA int32 tensor")
        p_host, p_ptr = 0, pos.data_ptr()
    else:
        p_host, p_ptr = int(pos), None
    fn = _native.lib().fqkv_quantize_int4_into_cache if int4 else _native.lib().fqkv_quantize_int8_into_cache
    with _DeviceGuard(dev):
        rc = fn(X.data_ptr(), codes.data_ptr(), scales.data_ptr(), G, T, D, cap, p_host, p_ptr, _stream(dev))
    _native.check(rc, f"launch: {op}")


def gqa_sk_fast(q, K, V, m_part, l_part, o_part, o, S, W, CW) -> None:
    """GQA split-K decode into caller buffers (batch 1).

    q [Hq,D] f16, K/V [Hkv,N,D] f16, scratch m_part/l_part [Hq,S] f32,
    o_part [Hq,S,D] f32, output o [Hq,D] f16.  Replaces ``gqa_sk_fast``
    (kernels/decode_attn_gqa_sk_fast.cu:95-112).  Scratch contents afterwards
    are unspecified.
    """
    op = "gqa_sk_fast"
    dev = _require_cuda(op, q, K, V, m_part, l_part, o_part, o)
    _require_dtype(op, "fp16", torch.float16, q=q, K=K, V=V, o=o)
    _require_dtype(op, "f32", torch.float32, m_part=m_part, l_part=l_part, o_part=o_part)
    _require_contig(op, q=q, K=K, V=V, m_part=m_part, l_part=l_part, o_part=o_part, o=o)
    _require_W(op, W)
    if int(CW) not in (4, 8):
        _fail(op, "CW", f"CW must be 4 or 8 (got {CW})")
    S = int(S)
    if S < 1:
        _fail(op, "S", f"S must be >= 1 (got {S})")
    if q.dim() != 2 or K.dim() != 3:
        _fail(op, "shape", "q must be [Hq, D] and K [Hkv, N, D]")
    Hq, D = q.shape
    Hkv, N, _ = K.shape
    _require_D(op, D)
    _require_shape(op, "K", K, (Hkv, N, D))
    _require_shape(op, "V", V, (Hkv, N, D))
    _require_shape(op, "m_part", m_part, (Hq, S))
    _require_shape(op, "l_part", l_part, (Hq, S))
    _require_shape(op, "o_part", o_part, (Hq, S, D))
    _require_shape(op, "o", o, (Hq, D))
    with _DeviceGuard(dev):
        rc = _native.lib().fqkv_gqa_sk_fast(
            q.data_ptr(), K.data_ptr(), V.data_ptr(), m_part.data_ptr(), l_part.data_ptr(), o_part.data_ptr(),
            o.data_ptr(), Hq, Hkv, N, D, S, int(W), int(CW), _stream(dev))
    _native.check(rc, f"launch: {op}")


def _quantize(op: str, X: torch.Tensor, int4: bool):
    dev = _require_cuda(op, X)
    _require_dtype(op, "fp16", torch.float16, X=X)
    _require_contig(op, X=X)
    if X.dim() < 1:
        _fail(op, "shape", "X must have a head_dim axis")
    D = X.shape[-1]
    if int4 and D % 2:
        _fail(op, "D", f"int4 packing needs an even head_dim (got {D})")
    rows = X.numel() // D if D else 0
    codes = torch.empty(X.shape[:-1] + ((D // 2,) if int4 else (D,)),
                        dtype=torch.uint8 if int4 else torch.int8, device=dev)
    scales = torch.empty(X.shape[:-1], dtype=torch.float16, device=dev)
    fn = _native.lib().fqkv_quantize_int4_per_token if int4 else _native.lib().fqkv_quantize_int8_per_token
    with _DeviceGuard(dev):
        rc = fn(X.data_ptr(), codes.data_ptr(), scales.data_ptr(), rows, D, _stream(dev))
    _native.check(rc, f"launch: {op}")
    return codes, scales


def decode_attn_kvcache_tp(q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, seq_len, tp,
                           Ks: torch.Tensor | None = None, Vs: torch.Tensor | None = None,
                           workspace: torch.Tensor | None = None) -> None:
    """Tensor-parallel decode step over this rank's KV cache, output sent to every rank.

    As :func:`decode_attn_gqa_kvcache` (fp16 cache, ``Ks``/``Vs`` None) or
    :func:`decode_attn_gqa_int8_kvcache` (int8 codes with their scales), but the
    [B, Hq, D] output is stored into every rank's receive buffer described by
    ``tp`` (a ``_native.TpOut``; see :class:`tp_exchange.PeerExchange`) and counted
    on every rank's arrival counters.  Returns nothing: the gathered outputs are
    read after :func:`tp_wait`.
    """
    op = "decode_attn_kvcache_tp"
    if Ks is None:
        dev = _require_cuda(op, q, K, V)
        _require_dtype(op, "fp16", torch.float16, q=q, K=K, V=V)
        _require_contig(op, q=q, K=K, V=V)
        if q.dim() != 3 or K.dim() != 4:
            _fail(op, "shape", "q must be [B, Hq, D] and K [B, Hkv, max_len, D]")
        B, Hq, D = q.shape
        _, Hkv, max_len, _ = K.shape
        _require_D(op, D)
        _require_shape(op, "K", K, (B, Hkv, max_len, D))
        _require_shape(op, "V", V, (B, Hkv, max_len, D))
        if Hkv < 1 or Hq % Hkv:
            _fail(op, "shape", f"Hq ({Hq}) must be a multiple of Hkv ({Hkv})")
        fmt = _native.KV_F16
    else:
        dev, B, Hq, Hkv, max_len, D = _check_int8_gqa(op, q, K, V, Ks, Vs)
        fmt = _native.KV_INT8
    n_host, n_ptr, _ = _seq_len_args(op, seq_len, dev, max_len)
    nb = workspace.numel() if workspace is not None else 0
    with _DeviceGuard(dev):
        rc = _native.lib().fqkv_decode_attn_kvcache_tp(
            fmt, q.data_ptr(), K.data_ptr(), V.data_ptr(), Ks.data_ptr() if Ks is not None else None,
            Vs.data_ptr() if Vs is not None else None, B, Hq, Hkv, max_len, D, n_host, n_ptr,
            workspace.data_ptr() if workspace is not None else None, nb, ctypes.byref(tp), _stream(dev))
    _native.check(rc, f"launch: {op}")


# Codes of the in-kernel status word (fqkv_device_status): the first bounded wait that gave up.
DEVICE_STATUS = {
    61: "a decode kernel's wait for a KV tile ran out",
    62: "a decode kernel's producer waited too long for a free pipeline stage",
    63: "a decode kernel could not drain its in-flight copies",
    64: "a tensor-parallel peer's attention outputs never arrived (a rank stopped or fell behind)",
}


def device_status(device: torch.device, clear: bool = True) -> int:
    """Reads (and by default resets) the in-kernel status word of ``device``: 0 when every
    bounded wait since the last reset completed, else the code of the first that gave up.
    Synchronizes with the device."""
    st = ctypes.c_int(-1)
    with _DeviceGuard(device):
        rc = _native.lib().fqkv_device_status(ctypes.byref(st), 1 if clear else 0)
    _native.check(rc, "device_status")
    return int(st.value)


def check_device_status(device: torch.device, what: str) -> None:
    """Raises RuntimeError when a bounded in-kernel wait on ``device`` gave up since the
    last check (the kernels then returned without their result instead of hanging); the
    status word is reset, so the next call on the device starts clean."""
    st = device_status(device, clear=True)
    if st != 0:
        raise RuntimeError(f"{what}: device status {st}: {DEVICE_STATUS.get(st, 'unknown code')}")


def tp_wait(counters_ptr: int, world: int, per_call: int, sequence_ptr: int, device: torch.device) -> None:
    """Enqueue the bounded wait for every rank's tensor-parallel outputs of one call (see the C ABI)."""
    with _DeviceGuard(device):
        rc = _native.lib().fqkv_tp_wait(counters_ptr, world, per_call, sequence_ptr, _stream(device))
    _native.check(rc, "launch: tp_wait")


def rope_qkv_append(qkv: torch.Tensor, cos_table: torch.Tensor, sin_table: torch.Tensor, pos,
                    q_out: torch.Tensor, K: torch.Tensor, V: torch.Tensor,
                    Ks: torch.Tensor | None = None, Vs: torch.Tensor | None = None) -> None:
    """Fused decode-step prologue: RoPE(q, k), q -> fp16, append k/v to the cache (see the C ABI).

    qkv [B, W] (fp16 or bf16, W >= (Hq + 2 Hkv) D, contiguous rows) holds each
    sequence's fused projection output [q heads | k heads | v heads];
    cos_table / sin_table [rows, D] are the model's rotary tables (same dtype);
    ``pos`` is an int or a CUDA int32 tensor (read on the device).  q_out
    [B, Hq, D] fp16; K/V [B, Hkv, cap, D] fp16 cache, or int8 codes with
    Ks/Vs [B, Hkv, cap] fp16 scales.  Bit-exact with transformers'
    apply_rotary_pos_emb, ``.to(float16)`` and (int8) :func:`qpt` of the new token.
    """
    op = "rope_qkv_append"
    dev = _require_cuda(op, qkv, cos_table, sin_table, q_out, K, V)
    if qkv.dtype not in (torch.float16, torch.bfloat16):
        _fail(op, "dtype", "qkv must be fp16 or bf16")
    _require_dtype(op, "model dtype", qkv.dtype, cos_table=cos_table, sin_table=sin_table)
    _require_dtype(op, "fp16", torch.float16, q_out=q_out)
    if qkv.dim() != 2 or qkv.stride(1) != 1 or q_out.dim() != 3 or K.dim() != 4:
        _fail(op, "shape", "qkv [B, W] with contiguous rows, q_out [B, Hq, D], K [B, Hkv, cap, D]")
    _require_contig(op, cos_table=cos_table, sin_table=sin_table, q_out=q_out, K=K, V=V)
    B, Hq, D = q_out.shape
    _, Hkv, cap, _ = K.shape
    _require_D(op, D)
    _require_shape(op, "V", V, (B, Hkv, cap, D))
    if cos_table.dim() != 2 or cos_table.shape[1] != D or sin_table.shape != cos_table.shape:
        _fail(op, "shape", "cos_table / sin_table must be [rows, D]")
    if Ks is None:
        _require_dtype(op, "fp16", torch.float16, K=K, V=V)
        fmt = _native.KV_F16
    else:
        _require_dtype(op, "int8", torch.int8, K=K, V=V)
        _require_dtype(op, "fp16", torch.float16, Ks=Ks, Vs=Vs)
        _require_contig(op, Ks=Ks, Vs=Vs)
        _require_shape(op, "Ks", Ks, (B, Hkv, cap))
        _require_shape(op, "Vs", Vs, (B, Hkv, cap))
        fmt = _native.KV_INT8
    if qkv.shape[0] != B or qkv.shape[1] < (Hq + 2 * Hkv) * D:
        _fail(op, "shape", f"qkv must be [B={B}, >= (Hq + 2 Hkv) D = {(Hq + 2 * Hkv) * D}]")
    if isinstance(pos, torch.Tensor):
        if pos.device != dev or pos.dtype != torch.int32 or pos.numel() < 1:
            _fail(op, "pos", "a tensor pos must be a CUDA int32 tensor on the inputs' device")
        pos_host, pos_ptr = 0, pos.data_ptr()
    else:
        pos_host, pos_ptr = int(pos), None
    with _DeviceGuard(dev):
        rc = _native.lib().fqkv_rope_qkv_append(
            fmt, 1 if qkv.dtype == torch.bfloat16 else 0, qkv.data_ptr(), qkv.stride(0), cos_table.data_ptr(),
            sin_table.data_ptr(), cos_table.shape[0], pos_host, pos_ptr, q_out.data_ptr(), K.data_ptr(),
            V.data_ptr(), Ks.data_ptr() if Ks is not None else None, Vs.data_ptr() if Vs is not None else None,
            B, Hq, Hkv, D, cap, _stream(dev))
    _native.check(rc, f"launch: {op}")


def add_rmsnorm(h: torch.Tensor, delta: torch.Tensor | None, weight: torch.Tensor, y: torch.Tensor,
                eps: float) -> None:
    """Residual add + RMSNorm in one launch: ``h += delta`` (if given, in place), ``y = rmsnorm(h) * weight``.

    h, delta, y [rows, H] and weight [H] in the model dtype (fp16 / bf16),
    contiguous; LlamaRMSNorm's arithmetic (fp32 inside, rounded to the model
    dtype where transformers rounds).
    """
    op = "add_rmsnorm"
    ts = dict(h=h, weight=weight, y=y) if delta is None else dict(h=h, delta=delta, weight=weight, y=y)
    dev = _require_cuda(op, *ts.values())
    if h.dtype not in (torch.float16, torch.bfloat16):
        _fail(op, "dtype", "h must be fp16 or bf16")
    _require_dtype(op, "model dtype", h.dtype, **ts)
    _require_contig(op, **ts)
    H = h.shape[-1]
    rows = h.numel() // H
    if weight.numel() != H or y.shape != h.shape or (delta is not None and delta.shape != h.shape):
        _fail(op, "shape", "h, delta, y [rows, H] and weight [H]")
    with _DeviceGuard(dev):
        rc = _native.lib().fqkv_add_rmsnorm(1 if h.dtype == torch.bfloat16 else 0, h.data_ptr(),
                                            delta.data_ptr() if delta is not None else None, weight.data_ptr(),
                                            y.data_ptr(), rows, H, float(eps), _stream(dev))
    _native.check(rc, f"launch: {op}")


def silu_mul(gu: torch.Tensor, y: torch.Tensor) -> None:
    """SwiGLU on a fused [gate | up] projection: gu [rows, 2I] -> y [rows, I] = silu(gate) * up (model dtype)."""
    op = "silu_mul"
    dev = _require_cuda(op, gu, y)
    if gu.dtype not in (torch.float16, torch.bfloat16):
        _fail(op, "dtype", "gu must be fp16 or bf16")
    _require_dtype(op, "model dtype", gu.dtype, y=y)
    _require_contig(op, y=y)
    if gu.dim() != 2 or gu.stride(1) != 1 or y.dim() != 2 or gu.shape[0] != y.shape[0] or gu.shape[1] < 2 * y.shape[1]:
        _fail(op, "shape", "gu [rows, >= 2I] with contiguous rows, y [rows, I]")
    with _DeviceGuard(dev):
        rc = _native.lib().fqkv_silu_mul(1 if gu.dtype == torch.bfloat16 else 0, gu.data_ptr(), y.data_ptr(),
                                         y.shape[0], y.shape[1], gu.stride(0), _stream(dev))
    _native.check(rc, f"launch: {op}")


def gemv(x: torch.Tensor, W: torch.Tensor, bias: torch.Tensor | None = None,
         out: torch.Tensor | None = None) -> torch.Tensor:
    """Small-batch projection y = x W^T (+ bias): x [B, K] (B <= 4), W [N, K], model dtype, fp32 accumulation.

    With bf16 weights x may be fp16 (rounded to bf16 as it is read, the same
    as ``x.to(torch.bfloat16)`` first); the output is in the weights' dtype.
    """
    op = "gemv"
    ts = dict(W=W) if bias is None else dict(W=W, bias=bias)
    dev = _require_cuda(op, x, *ts.values())
    if W.dtype not in (torch.float16, torch.bfloat16):
        _fail(op, "dtype", "W must be fp16 or bf16")
    _require_dtype(op, "model dtype", W.dtype, **ts)
    if x.dtype != W.dtype and x.dtype != torch.float16:
        _fail(op, "dtype", "x must be in the weights' dtype or fp16")
    _require_contig(op, x=x)
    _require_contig(op, **ts)
    if x.dim() != 2 or W.dim() != 2 or x.shape[1] != W.shape[1] or (bias is not None and bias.shape != (W.shape[0],)):
        _fail(op, "shape", "x [B, K], W [N, K], bias [N]")
    B, K = x.shape
    N = W.shape[0]
    if out is None:
        out = torch.empty(B, N, dtype=W.dtype, device=dev)
    code = {torch.float16: 0, torch.bfloat16: 1}
    with _DeviceGuard(dev):
        rc = _native.lib().fqkv_gemv(code[W.dtype], code[x.dtype], x.data_ptr(), W.data_ptr(),
                                     bias.data_ptr() if bias is not None else None, out.data_ptr(), B, N, K,
                                     _stream(dev))
    _native.check(rc, f"launch: {op}")
    return out


def gemv_swiglu(x: torch.Tensor, W: torch.Tensor, bias: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """A SwiGLU MLP's gate/up projection and the SwiGLU in one launch (small batch).

    x [B, K] (B <= 4), W [2I, K] = [gate_proj.weight; up_proj.weight], bias [2I] or None, all in
    the model dtype; returns y [B, I] = silu(g) * u with g, u the projections rounded to the model
    dtype -- the same values as ``silu_mul(gemv(x, W, bias), y)``.
    """
    op = "gemv_swiglu"
    ts = dict(x=x, W=W) if bias is None else dict(x=x, W=W, bias=bias)
    dev = _require_cuda(op, *ts.values())
    if W.dtype not in (torch.float16, torch.bfloat16):
        _fail(op, "dtype", "W must be fp16 or bf16")
    _require_dtype(op, "model dtype", W.dtype, **ts)
    _require_contig(op, **ts)
    if x.dim() != 2 or W.dim() != 2 or x.shape[1] != W.shape[1] or W.shape[0] % 2 \
            or (bias is not None and bias.shape != (W.shape[0],)):
        _fail(op, "shape", "x [B, K], W [2I, K], bias [2I]")
    B, K = x.shape
    I = W.shape[0] // 2
    if out is None:
        out = torch.empty(B, I, dtype=W.dtype, device=dev)
    elif out.shape != (B, I) or out.dtype != W.dtype or not out.is_contiguous():
        _fail(op, "out", "out must be a contiguous [B, I] tensor in the model dtype")
    with _DeviceGuard(dev):
        rc = _native.lib().fqkv_gemv_swiglu(1 if W.dtype == torch.bfloat16 else 0, x.data_ptr(), W.data_ptr(),
                                            bias.data_ptr() if bias is not None else None, out.data_ptr(), B, I, K,
                                            _stream(dev))
    _native.check(rc, f"launch: {op}")
    return out


def gemv_rope_append(x: torch.Tensor, W: torch.Tensor, bias: torch.Tensor | None, cos_table: torch.Tensor,
                     sin_table: torch.Tensor, pos, q_out: torch.Tensor, K: torch.Tensor, V: torch.Tensor) -> None:
    """Batch-1 q/k/v projection with RoPE, q -> fp16 and the k / v cache append in one launch.

    x [1, Hidden], W [(Hq + 2 Hkv) D, Hidden] (the concatenated q/k/v weights), bias or None, the
    rotary tables [rows, D] -- all in the model dtype; ``pos`` an int or a CUDA int32 tensor;
    q_out [1, Hq, D] fp16; K / V [1, Hkv, cap, D] fp16 caches.  The same values as
    ``rope_qkv_append(gemv(x, W, bias), cos_table, sin_table, pos, q_out, K, V)``.
    """
    op = "gemv_rope_append"
    ts = dict(x=x, W=W, cos_table=cos_table, sin_table=sin_table)
    if bias is not None:
        ts["bias"] = bias
    dev = _require_cuda(op, *ts.values(), q_out, K, V)
    if W.dtype not in (torch.float16, torch.bfloat16):
        _fail(op, "dtype", "W must be fp16 or bf16")
    _require_dtype(op, "model dtype", W.dtype, **ts)
    _require_dtype(op, "fp16", torch.float16, q_out=q_out, K=K, V=V)
    _require_contig(op, **ts)
    _require_contig(op, q_out=q_out, K=K, V=V)
    if x.dim() != 2 or x.shape[0] != 1 or q_out.dim() != 3 or q_out.shape[0] != 1 or K.dim() != 4 or K.shape[0] != 1:
        _fail(op, "shape", "x [1, Hidden], q_out [1, Hq, D], K / V [1, Hkv, cap, D]")
    _, Hq, D = q_out.shape
    _, Hkv, cap, _ = K.shape
    _require_D(op, D)
    _require_shape(op, "V", V, (1, Hkv, cap, D))
    if W.dim() != 2 or W.shape != ((Hq + 2 * Hkv) * D, x.shape[1]) or (bias is not None and bias.shape != (W.shape[0],)):
        _fail(op, "shape", f"W must be [(Hq + 2 Hkv) D = {(Hq + 2 * Hkv) * D}, {x.shape[1]}], bias [{W.shape[0]}]")
    if cos_table.dim() != 2 or cos_table.shape[1] != D or sin_table.shape != cos_table.shape:
        _fail(op, "shape", "cos_table / sin_table must be [rows, D]")
    if isinstance(pos, torch.Tensor):
        if pos.device != dev or pos.dtype != torch.int32 or pos.numel() < 1:
            _fail(op, "pos", "a tensor pos must be a CUDA int32 tensor on the inputs' device")
        pos_host, pos_ptr = 0, pos.data_ptr()
    else:
        pos_host, pos_ptr = int(pos), None
    with _DeviceGuard(dev):
        rc = _native.lib().fqkv_gemv_rope_append(
            1 if W.dtype == torch.bfloat16 else 0, x.data_ptr(), W.data_ptr(),
            bias.data_ptr() if bias is not None else None, x.shape[1], cos_table.data_ptr(), sin_table.data_ptr(),
            cos_table.shape[0], pos_host, pos_ptr, q_out.data_ptr(), K.data_ptr(), V.data_ptr(), Hq, Hkv, D, cap,
            _stream(dev))
    _native.check(rc, f"launch: {op}")


def argmax_rows(logits: torch.Tensor, scratch: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy choice per row: logits [rows, V] (fp16 / bf16) -> int64 [rows], as torch.argmax(-1).

    ``scratch``: a zero-filled uint8 tensor of ``fqkv_argmax_scratch_bytes(rows)``
    bytes, reusable across calls (and CUDA-graph replays).
    """
    op = "argmax_rows"
    dev = _require_cuda(op, logits, scratch)
    if logits.dtype not in (torch.float16, torch.bfloat16) or logits.dim() != 2 or logits.stride(1) != 1 \
            or logits.stride(0) != logits.shape[1]:
        _fail(op, "logits", "logits must be a contiguous fp16 / bf16 [rows, V] tensor")
    rows, V = logits.shape
    need = int(_native.lib().fqkv_argmax_scratch_bytes(rows))
    if scratch.dtype != torch.uint8 or scratch.numel() < need:
        _fail(op, "scratch", f"scratch must be a uint8 tensor of >= {need} bytes")
    if out is None:
        out = torch.empty(rows, dtype=torch.int64, device=dev)
    with _DeviceGuard(dev):
        rc = _native.lib().fqkv_argmax(1 if logits.dtype == torch.bfloat16 else 0, logits.data_ptr(), rows, V,
                                       scratch.data_ptr(), out.data_ptr(), _stream(dev))
    _native.check(rc, f"launch: {op}")
    return out


def qpt(X: torch.Tensor):
    """Per-token symmetric int8 quantizer: X [..., D] f16 -> (int8 [..., D], f16 scales [...]).

    Bit-exact with the reference's ``qpt`` (notebook lines 236-238,
    tests/test_kernels.py:32-34).
    """
    return _quantize("qpt", X, False)


def quant_int4_per_token(X: torch.Tensor):
    """Per-token symmetric int4 quantizer + packer: X [..., D] -> (uint8 [..., D/2], f16 [...]).

    Bit-exact with the reference's ``quant_int4_per_token`` (notebook lines
    292-299): element 2t in the low nibble of byte t.
    """
    return _quantize("quant_int4_per_token", X, True)
