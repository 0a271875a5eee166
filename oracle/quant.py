"""numpy restatement of the reference's per-token symmetric KV quantizers.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Reference algorithm (torch, all arithmetic on fp16 tensors):

* int8 ``qpt`` -- ``notebooks/integration_and_benchmarks.ipynb`` lines 236-238
  and ``tests/test_kernels.py:32-34``::

      a = |X|.amax(-1);  s = (a / 127).clamp(min=1e-8)
      codes = clamp(round(X / s), -127, 127).to(int8);  scales = s.half()

* int4 ``quant_int4_per_token`` -- notebook lines 292-299: the same with 7 in
  place of 127, then two signed nibbles per byte, element ``2t`` in the low
  nibble and ``2t+1`` in the high nibble (line 297-298).

* ``dequant_int4`` -- notebook lines 301-308: sign-extend each nibble
  (``x >= 8 -> x - 16``) and multiply by the fp32 scale.

fp16 semantics that make the codes bit-exact (verified against the
reference's own functions by ``tests/test_oracle_golden.py``):

1. ``a / 127`` on an fp16 tensor is computed in fp32 and rounded once to fp16.
   (torch CUDA multiplies by the fp32 reciprocal instead of dividing; for
   every finite non-negative fp16 ``a`` both give the same fp16 result for the
   divisors 127 and 7, which ``tests/test_oracle_golden.py`` checks
   exhaustively.)
2. ``clamp(min=1e-8)`` cannot raise a value: 1e-8 is below half the smallest
   fp16 subnormal, so an fp16 ``s`` is either 0 or already >= 1e-8 and the
   clamp only keeps NaN as NaN.  An all-zero token therefore has ``s = 0``.
3. ``X / s`` is fp16 / fp16: the fp32 IEEE quotient rounded to fp16.  The
   integer rounding ``round`` (half-to-even) is applied to that fp16 value, so
   the double rounding fp32 -> fp16 -> integer is part of the algorithm.
4. ``clamp`` keeps NaN; ``.to(int8)`` of NaN gives 0.  ``0/0`` (all-zero
   token) is NaN -> code 0; ``x/0`` for a nonzero x in a token whose scale
   underflowed to 0 is +-inf -> code +-127 (+-7).
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "quantize_int8_per_token",
    "quantize_int4_per_token",
    "pack_int4",
    "unpack_int4",
    "dequantize_int8",
    "dequantize_int4",
    "fp16_scale",
]


def fp16_scale(amax: np.ndarray, qmax: float) -> np.ndarray:
    """``(amax / qmax).clamp(min=1e-8)`` in fp16 tensor arithmetic (rules 1-2)."""
    amax = np.asarray(amax, dtype=np.float16)
    with np.errstate(invalid="ignore", over="ignore"):
        s = (amax.astype(np.float32) / np.float32(qmax)).astype(np.float16)
    # clamp(min=1e-8): 1e-8 rounds to fp16 zero; np.maximum keeps NaN.
    return np.maximum(s, np.float16(1e-8))


def _codes(X: np.ndarray, qmax: int) -> tuple[np.ndarray, np.ndarray]:
    X = np.asarray(X, dtype=np.float16)
    # amax over the last axis; NaN propagates like torch.amax.
    a = np.abs(X).max(axis=-1)
    s = fp16_scale(a, qmax)
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        r = (X.astype(np.float32) / s.astype(np.float32)[..., None]).astype(np.float16)
        r = np.rint(r.astype(np.float32))            # round half to even
        r = np.clip(r, -qmax, qmax)                   # NaN stays NaN
    codes = np.where(np.isnan(r), 0.0, r).astype(np.int8)
    return codes, s


def quantize_int8_per_token(X: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """``qpt``: X fp16 [..., D] -> (int8 codes [..., D], fp16 scales [...])."""
    return _codes(X, 127)


def pack_int4(codes: np.ndarray) -> np.ndarray:
    """Two's-complement nibbles, element 2t low, 2t+1 high (notebook 296-298)."""
    c = np.asarray(codes, dtype=np.int8)
    if c.shape[-1] % 2:
        raise ValueError("int4 packing needs an even head_dim")
    u = c.view(np.uint8) & np.uint8(0x0F)
    lo = u[..., 0::2]
    hi = u[..., 1::2]
    return (lo | (hi << np.uint8(4))).astype(np.uint8)


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """Inverse of :func:`pack_int4`: uint8 [..., D/2] -> int8 codes [..., D]."""
    b = np.asarray(packed, dtype=np.uint8).astype(np.int16)
    lo = b & 0xF
    hi = (b >> 4) & 0xF
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    out = np.empty(b.shape[:-1] + (b.shape[-1] * 2,), dtype=np.int8)
    out[..., 0::2] = lo
    out[..., 1::2] = hi
    return out


def quantize_int4_per_token(X: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """``quant_int4_per_token``: X fp16 [..., D] -> (uint8 [..., D/2], fp16 [...])."""
    codes, s = _codes(X, 7)
    return pack_int4(codes), s


def dequantize_int8(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """``Kq.float() * Ks.float()[..., None]`` (tests/test_kernels.py:37) in fp32."""
    with np.errstate(invalid="ignore"):
        return np.asarray(codes, np.int8).astype(np.float32) * \
        np.asarray(scales, np.float16).astype(np.float32)[..., None]


def dequantize_int4(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """``dequant_int4`` (notebook 301-308): sign-extended nibbles times fp32 scale."""
    with np.errstate(invalid="ignore"):
        return unpack_int4(packed).astype(np.float32) * \
            np.asarray(scales, np.float16).astype(np.float32)[..., None]
