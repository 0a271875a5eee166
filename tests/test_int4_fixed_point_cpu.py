"""CPU checks of the fixed-point arithmetic behind the int4 decode kernel's
integer P.V (``csrc/attn_qtc.cu``, one-head variant).

The kernel writes p * vscale as v = rint(p * vs * Ps) and splits it into
three 8-bit planes read straight out of the float 2^23 + 32896 + v (one FMA
with the magic constant): byte 2 is h, bytes 1 and 0 (xor 0x80) are the
signed m and l, v = h * 65536 + m * 256 + l.  The integer sums of one
"frame" (one reference maximum, one scale) are flushed to fp32 and rescaled
when the maximum grows by more than 2^headroom (log2) or when a tile's
largest p * vs would leave the fixed-point range.

These tests pin (1) the plane decomposition for every value the kernel can
produce, with the constants read from the kernel source, and (2) a numpy
model of the frame rules against float64 attention on adversarial inputs
(moving maxima, scale outliers, zero scales, masked keys).  They check the
arithmetic the kernel relies on; the kernel itself is checked on the GPU by
``test_parity_gpu.py``.
"""
from __future__ import annotations

import pathlib
import re

import numpy as np
import pytest

SRC = pathlib.Path(__file__).resolve().parents[1] / "fused-quantized-kv-decode-attention_b200" / "csrc" / "attn_qtc.cu"


def _const(name: str) -> float:
    m = re.search(rf"constexpr (?:float|int) {name} = ([0-9.e+-]+)f?;", SRC.read_text())
    assert m, name
    return float(m.group(1))


MAGIC = _const("kG1Magic")
HEADROOM = _const("kG1Headroom")
VLIM = _const("kG1VLim")
FRAME_TILES = int(_const("kG1FrameTiles"))


def _planes(v: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """The three planes as the kernel reads them out of fp32(MAGIC + v)."""
    bits = (np.float32(MAGIC) + v.astype(np.float32)).view(np.uint32)
    h = ((bits >> 16) & 0xFF).astype(np.int64)
    m = (((bits >> 8) & 0xFF) ^ 0x80).astype(np.uint8).view(np.int8).astype(np.int64)
    low = ((bits & 0xFF) ^ 0x80).astype(np.uint8).view(np.int8).astype(np.int64)
    return h, m, low


def test_magic_constant_and_range():
    assert MAGIC == 2.0 ** 23 + 32896
    assert VLIM <= 2 ** 23 - 1 - 32896          # u = v + 32896 stays below 2^23
    # s32 bound: |code term| <= 128 and |plane| <= 128 per key, 32 keys per tile and warp
    assert FRAME_TILES * 32 * 128 * 128 < 2 ** 31


def test_planes_reassemble_every_value():
    v = np.arange(0, int(VLIM) + 1, dtype=np.int64)
    h, m, low = _planes(v)
    assert h.min() >= 0 and h.max() <= 127
    assert np.array_equal(h * 65536 + m * 256 + low, v)


def test_fma_rounds_to_nearest_integer():
    rng = np.random.default_rng(0)
    x = rng.uniform(0, VLIM, 200_000)
    v = np.rint(x)
    got = (np.float64(MAGIC) + x).astype(np.float32).astype(np.float64) - MAGIC  # one rounding, as the FMA
    assert np.array_equal(got, v)


def _frames(s, vs, codes, valid, tile=32):
    """The kernel's frame rules for one warp's keys (tiles of 32 keys)."""
    n, d = codes.shape
    acc = np.zeros((d, 3), np.int64)
    bs = np.zeros(3, np.int64)
    o = np.zeros(d)
    lsum, m_run, ps, inv_ps, ft, frames = 0.0, -np.inf, 0.0, 0.0, 0, 0
    low = np.arange(d) % 2 == 0                       # even dims: low nibbles, entered as code + 8
    bias = np.where(low, 8, 0)
    unit = np.where(low, 1.0, 1.0 / 16)               # odd dims: high nibbles, entered as 16 * code

    def flush(rescale):
        nonlocal o
        x = (acc[:, 0] - bias * bs[0]) * 65536.0 + (acc[:, 1] - bias * bs[1]) * 256.0 + (acc[:, 2] - bias * bs[2])
        o = (x * unit * inv_ps + o) * rescale
        acc[:] = 0
        bs[:] = 0

    for t0 in range(0, n, tile):
        sl = slice(t0, t0 + tile)
        st, vt, ct, ok = s[sl], vs[sl], codes[sl], valid[sl]
        mx = st[ok].max() if ok.any() else -np.inf
        if mx > m_run + HEADROOM:
            rescale = 0.0 if m_run == -np.inf else 2.0 ** (m_run - mx)
            flush(rescale)
            lsum *= rescale
            m_run, ft = mx, 0
            frames += 1
        p = np.where(ok, 2.0 ** (st - m_run), 0.0).astype(np.float32) if m_run > -np.inf else np.zeros(len(st), np.float32)
        pv = (p * vt).astype(np.float32)
        pvm = float(pv.max())
        if pvm * ps > VLIM or ft >= FRAME_TILES or (ps == 0.0 and pvm > 0.0):
            flush(1.0)
            ft = 0
            frames += 1
            if pvm > 0.0:
                pb = 1.25 * max(pvm, 1e-30)
                ps, inv_ps = np.float32(VLIM / pb), pb / VLIM
        ft += 1
        v = np.rint(pv.astype(np.float64) * np.float64(ps))
        assert v.max() <= VLIM
        h, m, lo = _planes(v)
        planes = np.stack([h, m, lo], 1) * ok[:, None]
        bs += planes.sum(0)
        field = np.where(low[None, :], ct + 8, 16 * ct)
        acc += field.T @ planes
        lsum += float(p.sum())
    flush(1.0)
    return o / lsum, frames


@pytest.mark.parametrize("case", ["random", "moving_max", "scale_outliers", "peaked_and_outliers"])
def test_frames_match_float64_attention(case):
    rng = np.random.default_rng({"random": 1, "moving_max": 2, "scale_outliers": 3, "peaked_and_outliers": 4}[case])
    n, d = 2048, 8
    s = rng.normal(0, 1.44, n)
    vs = rng.uniform(0.3, 0.6, n).astype(np.float32)
    if case == "moving_max":
        s = s + np.linspace(0, 60, n)                 # the maximum moves by more than 2^3 again and again
    if case in ("scale_outliers", "peaked_and_outliers"):
        vs[rng.integers(0, n, 4)] *= 100
        vs[500:700] *= 1e-3
        vs[900] = 0
    if case == "peaked_and_outliers":
        s = rng.normal(0, 7.0, n)
    codes = rng.integers(-7, 8, (n, d))
    valid = rng.random(n) < 0.95
    got, frames = _frames(s, vs, codes, valid)
    w = np.where(valid, 2.0 ** (s - s[valid].max()), 0.0)
    ref = (w[:, None] * vs[:, None] * codes).sum(0) / w.sum()
    assert frames >= 2
    np.testing.assert_allclose(got, ref, atol=2e-4 * max(1.0, np.abs(ref).max()), rtol=1e-3)
