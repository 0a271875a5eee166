"""CPU emulation of one warp tile of the int4 decode kernel's integer P.V
(``csrc/attn_qtc.cu``, one-head variant): the k-slot -> key map ``g1_key``,
the per-lane ldmatrix row addresses, the byte permutes that turn ldmatrix.trans
pairs into four-key A registers, the three-plane P packing and its shuffle
sources, against a direct sum.  The fragment layouts are the documented PTX
ones (mma.m16n8k32 with 8-bit operands, ldmatrix.m8n8.x4.trans.b16).  Also
checks that every ldmatrix 8x8 matrix reads 8 rows that differ mod 8 (no bank
conflicts under the 64-byte swizzle) and that the K-side loads of neighbouring
lane groups alternate row parity.  Any k-slot -> key bijection used on both
sides gives a correct product; what singles out ``g1_key`` is the bank-conflict
freedom, which the second test pins (the naive map 8i + g fails it), while the
tile test guards the fragment layouts, permutes, plane packing and shuffle
sources.  The kernel itself is checked on the GPU by ``test_parity_gpu.py``."""
from __future__ import annotations

import pathlib

import numpy as np

SRC = pathlib.Path(__file__).resolve().parents[1] / "fused-quantized-kv-decode-attention_b200" / "csrc" / "attn_qtc.cu"
D, RB, KPW = 128, 64, 32
MAGIC = np.float32(8421504.0)


def g1_key(g: int, i: int) -> int:
    return 8 * i + (g ^ (4 * (i & 1)))


def prmt(a: int, b: int, sel: int) -> int:
    by = [(a >> (8 * k)) & 0xFF for k in range(4)] + [(b >> (8 * k)) & 0xFF for k in range(4)]
    return sum(by[(sel >> (4 * k)) & 7] << (8 * k) for k in range(4))


def s8(x: int) -> int:
    return x - 256 if x >= 128 else x


def bytes_of(w: int) -> list[int]:
    return [(w >> (8 * k)) & 0xFF for k in range(4)]


def test_source_uses_the_same_key_map():
    assert "return 8 * i + (g ^ (4 * (i & 1)));" in SRC.read_text()


def test_key_map_is_a_bijection_and_conflict_free():
    assert sorted(g1_key(a, i) for a in range(8) for i in range(4)) == list(range(32))
    for L0 in range(0, 32, 8):                      # one ldmatrix 8x8 matrix per 8 lanes
        rows = [_ldsm_row(L) for L in range(L0, L0 + 8)]
        assert len({r % 8 for r in rows}) == 8
    for i in range(4):                              # K loads: lane groups 2j, 2j+1 in one phase
        for j in range(4):
            assert (g1_key(2 * j, i) - g1_key(2 * j + 1, i)) % 2 == 1


def _ldsm_row(L: int) -> int:
    mi, rr = L >> 3, L & 7
    return g1_key((rr >> 1) + 4 * (mi >> 1), 2 * (mi & 1) + (rr & 1))


def test_one_warp_tile_matches_a_direct_sum():
    rng = np.random.default_rng(0)
    codes = rng.integers(-7, 8, size=(KPW, D))
    packed = ((codes[:, 0::2] & 0xF) | ((codes[:, 1::2] & 0xF) << 4)).astype(np.uint8)
    smem = np.zeros(KPW * RB, np.uint8)             # 64-byte rows, chunk c at c ^ ((row >> 1) & 3)
    for r in range(KPW):
        for c in range(4):
            cc = c ^ ((r >> 1) & 3)
            smem[r * RB + cc * 16:r * RB + cc * 16 + 16] = packed[r, c * 16:(c + 1) * 16]
    valid = rng.random(KPW) < 0.9
    p = np.where(valid, 2.0 ** rng.uniform(-6, 3, KPW), 0.0).astype(np.float32)
    vs = rng.uniform(0.3, 0.6, KPW).astype(np.float32)
    pv = (p * vs).astype(np.float32)
    ps = np.float32(8.0e6 / (1.25 * pv.max()))

    # P planes: lane (g, t < 3) packs plane t of keys g1_key(g, 0..3); B fragment by two shuffles
    W = [0] * 32
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        fw = [int(np.float32(np.float64(pv[g1_key(g, i)]) * np.float64(ps) + np.float64(MAGIC)).view(np.uint32))
              for i in range(4)]
        b = 2 if t == 0 else (1 if t == 1 else 0)
        psel = b | ((4 + b) << 4)
        pxor = 0x80808080 if t in (1, 2) else 0
        pmask = 0xFFFFFFFF if t < 3 else 0
        W[lane] = (prmt(prmt(fw[0], fw[1], psel), prmt(fw[2], fw[3], psel), 0x5410) ^ pxor) & pmask
    Bm = np.zeros((32, 8), np.int64)                # B[k-slot][column]
    for lane in range(32):
        g, t = lane >> 2, lane & 3
        b0, b1 = W[4 * t + (g & 3)], W[16 + 4 * t + (g & 3)]
        for i in range(4):
            Bm[4 * t + i, g] = s8(bytes_of(b0)[i])
            Bm[16 + 4 * t + i, g] = s8(bytes_of(b1)[i])
    for s in range(32):                             # slot 4a + i carries key g1_key(a, i)
        v = Bm[s, 0] * 65536 + Bm[s, 1] * 256 + Bm[s, 2]
        assert v == int(np.rint(np.float64(pv[g1_key(s >> 2, s & 3)]) * np.float64(ps)))

    # V fragments: ldmatrix.x4.trans per 16-byte segment, two byte permutes per register pair
    acc = np.zeros((8, 16, 8), np.int64)            # m-tile, row, column
    for sg in range(4):
        rows = []
        for L in range(32):
            r = _ldsm_row(L)
            off = (r * RB) | (((r >> 1) & 3) << 4)
            rows.append([int(x) for x in smem[(off ^ (sg << 4)):(off ^ (sg << 4)) + 16]])
        A_lo = np.zeros((16, 32), np.int64)
        A_hi = np.zeros((16, 32), np.int64)
        for lane in range(32):
            g, t = lane >> 2, lane & 3
            vr = []
            for m in range(4):                      # thread (g, t) gets rows 2t, 2t+1, b16 column g
                r0, r1 = rows[8 * m + 2 * t], rows[8 * m + 2 * t + 1]
                vr.append(r0[2 * g] | (r0[2 * g + 1] << 8) | (r1[2 * g] << 16) | (r1[2 * g + 1] << 24))
            w = [prmt(vr[0], vr[1], 0x6420), prmt(vr[0], vr[1], 0x7531),
                 prmt(vr[2], vr[3], 0x6420), prmt(vr[2], vr[3], 0x7531)]
            for k in range(4):                      # a0: row g, k 4t+i; a1: row g+8; a2/a3: k + 16
                for reg, (row, kk) in enumerate(((g, 4 * t), (g + 8, 4 * t), (g, 16 + 4 * t), (g + 8, 16 + 4 * t))):
                    A_lo[row, kk + k] = bytes_of((w[reg] ^ 0x08080808) & 0x0F0F0F0F)[k]
                    A_hi[row, kk + k] = s8(bytes_of(w[reg] & 0xF0F0F0F0)[k])
        acc[sg] += A_lo @ Bm
        acc[4 + sg] += A_hi @ Bm
    bs = [sum(Bm[:, c]) for c in range(3)]          # the + 8 of the low nibbles
    O = np.zeros(D)
    for g in range(8):
        for sg in range(4):
            lo = lambda r: (acc[sg, r, 0] - 8 * bs[0]) * 65536 + (acc[sg, r, 1] - 8 * bs[1]) * 256 + acc[sg, r, 2] - 8 * bs[2]
            hi = lambda r: (acc[4 + sg, r, 0] * 65536 + acc[4 + sg, r, 1] * 256 + acc[4 + sg, r, 2]) / 16
            O[32 * sg + 4 * g:32 * sg + 4 * g + 4] = [lo(g), hi(g), lo(g + 8), hi(g + 8)]
    O /= float(ps)
    ref = (pv[:, None].astype(np.float64) * codes).sum(0)
    np.testing.assert_allclose(O, ref, atol=2e-6 * np.abs(ref).max())
