"""Pin the CPU oracle against the reference's own outputs (CPU only).

The golden vectors in ``tests/golden/*.npz`` were produced by executing the
reference's Python functions (``tests/golden/make_golden.py``).  The numpy
restatement in ``oracle/`` must reproduce the quantizer bit-exactly and the
attention outputs within the build's tolerance.
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import attention as oatt
from oracle import quant as oq

ATOL, RTOL = 2e-3, 1e-2


@pytest.fixture(scope="module")
def qg(golden_dir):
    return dict(np.load(golden_dir / "quant_golden.npz"))


@pytest.fixture(scope="module")
def ag(golden_dir):
    return dict(np.load(golden_dir / "attention_golden.npz"))


def _same_fp16(a, b):
    a = np.asarray(a, np.float16)
    b = np.asarray(b, np.float16)
    both_nan = np.isnan(a) & np.isnan(b)
    return np.array_equal(a.view(np.uint16)[~both_nan], b.view(np.uint16)[~both_nan]) and \
        np.array_equal(np.isnan(a), np.isnan(b))


@pytest.mark.parametrize("tag", ["rand", "edge"])
@pytest.mark.parametrize("D", [64, 128])
def test_int8_quantizer_bit_exact(qg, tag, D):
    X = qg[f"X_{tag}_D{D}"]
    codes, scales = oq.quantize_int8_per_token(X)
    assert np.array_equal(codes, qg[f"codes8_{tag}_D{D}"])
    assert _same_fp16(scales, qg[f"scales8_{tag}_D{D}"])


@pytest.mark.parametrize("tag", ["rand", "edge"])
@pytest.mark.parametrize("D", [64, 128])
def test_int4_quantizer_bit_exact(qg, tag, D):
    X = qg[f"X_{tag}_D{D}"]
    packed, scales = oq.quantize_int4_per_token(X)
    assert np.array_equal(packed, qg[f"packed4_{tag}_D{D}"])
    assert _same_fp16(scales, qg[f"scales4_{tag}_D{D}"])
    deq = oq.dequantize_int4(packed, scales)
    ref = qg[f"deq4_{tag}_D{D}"]
    assert np.array_equal(np.isnan(deq), np.isnan(ref))
    m = ~np.isnan(ref)
    assert np.array_equal(deq[m], ref[m])


def test_int4_pack_round_trip():
    rng = np.random.default_rng(0)
    codes = rng.integers(-8, 8, size=(5, 11, 128)).astype(np.int8)
    assert np.array_equal(oq.unpack_int4(oq.pack_int4(codes)), codes)


# The reference records int4 accuracy against true fp32 attention as
# max|int4 - fp32| / max|fp32| = 0.145 / 0.227 / 0.180 for (B, N) = (8, 1024),
# (8, 4096), (64, 2048), D = 64, N(0,1) inputs (notebook lines 447-449, computed
# at lines 476-485; "about 15 to 23 %").  Its inputs were drawn on a GPU and
# cannot be reproduced here, so the pin is the band: the oracle's int4 path (the
# GPU kernels match it within 2e-3) on seeded CPU draws of the same shapes.
@pytest.mark.parametrize("B,N,recorded", [(8, 1024, 0.14545), (8, 4096, 0.22689), (64, 2048, 0.17994)])
def test_int4_accuracy_vs_fp32_in_the_recorded_band(B, N, recorded):
    import torch
    g = torch.Generator().manual_seed(0)
    q = torch.randn(B, 64, generator=g).half().numpy()
    K = torch.randn(B, N, 64, generator=g).half().numpy()
    V = torch.randn(B, N, 64, generator=g).half().numpy()
    Kp, Ks = oq.quantize_int4_per_token(K)
    Vp, Vs = oq.quantize_int4_per_token(V)
    out = oatt.decode_attention(q, oq.dequantize_int4(Kp, Ks), oq.dequantize_int4(Vp, Vs))
    ref = oatt.decode_attention(q, K, V)
    rel = np.abs(out - ref).max() / np.abs(ref).max()
    assert 0.5 * 0.145 < rel < 2.0 * 0.227, (rel, recorded)


@pytest.mark.parametrize("qmax", [127.0, 7.0])
def test_scale_division_rule_exhaustive(qmax):
    """fp32 division and torch-CUDA's multiply-by-reciprocal agree on every fp16."""
    a = np.arange(0, 0x7C00, dtype=np.uint16).view(np.float16)
    div = (a.astype(np.float32) / np.float32(qmax)).astype(np.float16)
    mul = (a.astype(np.float32) * (np.float32(1.0) / np.float32(qmax))).astype(np.float16)
    assert np.array_equal(div.view(np.uint16), mul.view(np.uint16))
    assert np.array_equal(oq.fp16_scale(a, qmax).view(np.uint16), div.view(np.uint16))


def _row_keys(ag):
    return sorted(k[2:] for k in ag if k.startswith("q_R"))


def test_attention_oracle_matches_reference_cpu_path(ag):
    for key in _row_keys(ag):
        q, K, V = ag[f"q_{key}"], ag[f"K_{key}"], ag[f"V_{key}"]
        o = oatt.decode_attention(q, K, V)
        np.testing.assert_allclose(o, ag[f"einsum_{key}"], atol=1e-5, rtol=1e-5)
        np.testing.assert_allclose(o, ag[f"sdpa_{key}"].astype(np.float64), atol=ATOL, rtol=RTOL)
        np.testing.assert_allclose(o, ag[f"sdparef_{key}"].astype(np.float64), atol=ATOL, rtol=RTOL)


def test_quantized_attention_oracle_matches_reference(ag):
    for key in _row_keys(ag):
        q, K, V = ag[f"q_{key}"], ag[f"K_{key}"], ag[f"V_{key}"]
        Kq, Ks = oq.quantize_int8_per_token(K)
        Vq, Vs = oq.quantize_int8_per_token(V)
        o8 = oatt.decode_attention(q, oq.dequantize_int8(Kq, Ks), oq.dequantize_int8(Vq, Vs))
        np.testing.assert_allclose(o8, ag[f"int8ref_{key}"].astype(np.float64), atol=ATOL, rtol=RTOL)
        Kp, Ks4 = oq.quantize_int4_per_token(K)
        Vp, Vs4 = oq.quantize_int4_per_token(V)
        o4 = oatt.decode_attention(q, oq.dequantize_int4(Kp, Ks4), oq.dequantize_int4(Vp, Vs4))
        np.testing.assert_allclose(o4, ag[f"int4ref_{key}"].astype(np.float64), atol=ATOL, rtol=RTOL)


def test_gqa_oracle_matches_reference(ag):
    keys = sorted(k[2:] for k in ag if k.startswith("q_gqa"))
    assert keys
    for key in keys:
        o = oatt.decode_attention_gqa(ag[f"q_{key}"], ag[f"K_{key}"], ag[f"V_{key}"])
        np.testing.assert_allclose(o, ag[f"sdpa_{key}"].astype(np.float64), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("N,S", [(1024, 8), (3, 8), (1, 4), (100, 7), (37, 37)])
def test_splitk_algebra_matches_full_softmax(N, S):
    """The split/merge restatement equals one-pass attention, empty splits included."""
    rng = np.random.default_rng(N * 31 + S)
    Hq, Hkv, D = 32, 8, 64
    q = rng.standard_normal((Hq, D)).astype(np.float16)
    K = rng.standard_normal((Hkv, N, D)).astype(np.float16)
    V = rng.standard_normal((Hkv, N, D)).astype(np.float16)
    m, l, o = oatt.splitk_partials(q, K, V, S)
    out = oatt.splitk_combine(m, l, o)
    ref = oatt.decode_attention_gqa(q[None], K[None], V[None])[0]
    np.testing.assert_allclose(out, ref, atol=1e-9, rtol=1e-9)
