"""C-ABI checks that need no GPU: the library loads, exports exactly the
symbols ``include/fqkv_b200.h`` declares, and rejects bad arguments with the
reference's error conditions before touching CUDA."""
from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "fqkv_b200.h"


def header_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\*?\s+\*?(fqkv_[a-z0-9_]+)\s*\(", text, re.M))


def test_header_declares_expected_entry_points():
    syms = header_symbols()
    for name in ("fqkv_decode_attn_fp16_mw", "fqkv_decode_attn_int8_mw", "fqkv_decode_attn_int4",
                 "fqkv_decode_attn_gqa", "fqkv_gqa_sk_fast", "fqkv_quantize_int8_per_token",
                 "fqkv_quantize_int4_per_token", "fqkv_last_error", "fqkv_decode_workspace_bytes"):
        assert name in syms


def test_library_exports_every_header_symbol(fqkv):
    lib = fqkv.native.lib()
    for name in header_symbols():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert set(fqkv.native.SIGNATURES) == header_symbols()


def test_version(fqkv):
    assert b"sm_100a" in fqkv.native.lib().fqkv_version()


def _call(fqkv, name, *args):
    lib = fqkv.native.lib()
    rc = getattr(lib, name)(*args)
    return rc, fqkv.native.last_error()


P = ctypes.c_void_p(16)      # non-null, 16-byte aligned dummy (never dereferenced)
P3 = ctypes.c_void_p(18)     # 2-byte aligned only


@pytest.mark.parametrize("W", [0, 1, 3, 16])
def test_bad_W_rejected(fqkv, W):
    rc, msg = _call(fqkv, "fqkv_decode_attn_fp16_mw", P, P, P, P, 4, 16, 64, W, None, 0, None)
    assert rc == fqkv.native.ERR_INVALID_ARGUMENT and msg.startswith("W")


@pytest.mark.parametrize("D", [32, 96, 256])
def test_bad_D_rejected(fqkv, D):
    rc, msg = _call(fqkv, "fqkv_decode_attn_int8_mw", P, P, P, P, P, P, 4, 16, D, 8, None, 0, None)
    assert rc == fqkv.native.ERR_INVALID_ARGUMENT and msg.startswith("D")


def test_bad_CW_and_S_rejected(fqkv):
    f = "fqkv_gqa_sk_fast"
    rc, msg = _call(fqkv, f, P, P, P, P, P, P, P, 32, 8, 128, 64, 8, 8, 2, None)
    assert rc == fqkv.native.ERR_INVALID_ARGUMENT and msg.startswith("CW")
    rc, msg = _call(fqkv, f, P, P, P, P, P, P, P, 32, 8, 128, 64, 0, 8, 4, None)
    assert rc == fqkv.native.ERR_INVALID_ARGUMENT and msg.startswith("S")


def test_gqa_head_ratio_rejected(fqkv):
    rc, msg = _call(fqkv, "fqkv_decode_attn_gqa", P, P, P, P, 1, 6, 4, 16, 64, 8, None, 0, None)
    assert rc == fqkv.native.ERR_INVALID_ARGUMENT and "multiple" in msg


def test_empty_kv_rejected_and_empty_batch_is_noop(fqkv):
    rc, msg = _call(fqkv, "fqkv_decode_attn_fp16_mw", P, P, P, P, 4, 0, 64, 8, None, 0, None)
    assert rc == fqkv.native.ERR_INVALID_ARGUMENT and msg.startswith("N")
    rc, _ = _call(fqkv, "fqkv_decode_attn_fp16_mw", None, None, None, None, 0, 16, 64, 8, None, 0, None)
    assert rc == fqkv.native.OK


def test_misaligned_kv_rejected(fqkv):
    rc, msg = _call(fqkv, "fqkv_decode_attn_int4", P, P3, P, P, P, P, 4, 16, 64, 8, None, 0, None)
    assert rc == fqkv.native.ERR_MISALIGNED


def test_null_pointer_rejected(fqkv):
    rc, _ = _call(fqkv, "fqkv_decode_attn_int4", P, P, P, None, P, P, 4, 16, 64, 8, None, 0, None)
    assert rc == fqkv.native.ERR_INVALID_ARGUMENT


def test_int4_quantizer_odd_dim_rejected(fqkv):
    rc, msg = _call(fqkv, "fqkv_quantize_int4_per_token", P, P, P, 4, 63, None)
    assert rc == fqkv.native.ERR_INVALID_ARGUMENT and msg.startswith("D")


def test_python_layer_errors_match_reference_keywords(fqkv):
    import torch
    q = torch.zeros(2, 64, dtype=torch.float16)
    K = torch.zeros(2, 8, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="^cuda"):
        fqkv.decode_attn_fp16_mw(q, K, K, 8)
    with pytest.raises(RuntimeError, match="^cuda"):
        fqkv.qpt(K)


def test_workspace_query_without_gpu_is_zero(fqkv):
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present: the query returns a real size")
    assert fqkv.native.lib().fqkv_decode_workspace_bytes(0, 64, 32, 8, 16384, 128) == 0


def test_decode_step_kernels_reject_bad_arguments(fqkv):
    """The decode-step entries (GEMV, GEMV + SwiGLU, GEMV + RoPE + append, argmax, SwiGLU, add+RMSNorm)
    validate before launching."""
    bad, mis, ok = fqkv.native.ERR_INVALID_ARGUMENT, fqkv.native.ERR_MISALIGNED, fqkv.native.OK
    # GEMV: batch above 4, K not a multiple of 256, bf16 activations with fp16 weights, misaligned weights
    assert _call(fqkv, "fqkv_gemv", 1, 1, P, P, None, P, 5, 16, 256, None)[0] == bad
    assert _call(fqkv, "fqkv_gemv", 1, 1, P, P, None, P, 1, 16, 300, None)[0] == bad
    assert _call(fqkv, "fqkv_gemv", 0, 1, P, P, None, P, 1, 16, 256, None)[0] == bad
    assert _call(fqkv, "fqkv_gemv", 1, 1, P, P3, None, P, 1, 16, 256, None)[0] == mis
    # argmax: unknown dtype, more rows than the grid takes, empty rows, misaligned index output; no rows is a no-op
    assert _call(fqkv, "fqkv_argmax", 2, P, 1, 10, P, P, None)[0] == bad
    assert _call(fqkv, "fqkv_argmax", 1, P, 70000, 10, P, P, None)[0] == bad
    assert _call(fqkv, "fqkv_argmax", 1, P, 1, 0, P, P, None)[0] == bad
    assert _call(fqkv, "fqkv_argmax", 1, P, 1, 10, P, P3, None)[0] == mis
    assert _call(fqkv, "fqkv_argmax", 1, None, 0, 10, None, None, None)[0] == ok
    lib = fqkv.native.lib()
    assert lib.fqkv_argmax_scratch_bytes(0) == 0
    assert 0 < lib.fqkv_argmax_scratch_bytes(1) < lib.fqkv_argmax_scratch_bytes(64)
    # SwiGLU: a row stride shorter than the gate and up halves
    assert _call(fqkv, "fqkv_silu_mul", 1, P, P, 2, 100, 150, None)[0] == bad
    # GEMV + SwiGLU: batch above 4, K not a multiple of 256, unknown dtype, misaligned x
    assert _call(fqkv, "fqkv_gemv_swiglu", 1, P, P, None, P, 5, 16, 256, None)[0] == bad
    assert _call(fqkv, "fqkv_gemv_swiglu", 1, P, P, None, P, 1, 16, 300, None)[0] == bad
    assert _call(fqkv, "fqkv_gemv_swiglu", 2, P, P, None, P, 1, 16, 256, None)[0] == bad
    assert _call(fqkv, "fqkv_gemv_swiglu", 1, P3, P, None, P, 1, 16, 256, None)[0] == mis
    # GEMV + RoPE + append: head size 96, K not a multiple of 256, position outside the table, misaligned W
    assert _call(fqkv, "fqkv_gemv_rope_append", 1, P, P, None, 256, P, P, 10, 0, None, P, P, P, 8, 2, 96, 10,
                 None)[0] == bad
    assert _call(fqkv, "fqkv_gemv_rope_append", 1, P, P, None, 300, P, P, 10, 0, None, P, P, P, 8, 2, 64, 10,
                 None)[0] == bad
    assert _call(fqkv, "fqkv_gemv_rope_append", 1, P, P, None, 256, P, P, 10, 10, None, P, P, P, 8, 2, 64, 10,
                 None)[0] == bad
    assert _call(fqkv, "fqkv_gemv_rope_append", 1, P, P3, None, 256, P, P, 10, 0, None, P, P, P, 8, 2, 64, 10,
                 None)[0] == mis
    # add + RMSNorm: hidden size above 8192, odd address
    assert _call(fqkv, "fqkv_add_rmsnorm", 1, P, None, P, P, 2, 9000, 1e-5, None)[0] == bad
    assert _call(fqkv, "fqkv_add_rmsnorm", 1, ctypes.c_void_p(17), None, P, P, 2, 64, 1e-5, None)[0] == mis
