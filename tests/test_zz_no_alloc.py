"""The split-K entry point for callers that cannot allocate device memory.

Some callers may not call cudaMalloc where they run the op: a serving
runtime's enqueue/plugin hook that owns all device memory, a decode loop that
must not stall on an allocation, a C host without an allocator.  For them
``fqkv_gqa_sk_fast_static_scratch`` keeps the split partials in a fixed
4 MiB array inside the library instead of caller scratch.  This test calls it
through the C ABI twice in a row (different shapes, so stale contents of the
shared array from the first call must not leak into the second) and compares
each result with the float64 oracle and with the existing ``fqkv_gqa_sk_fast``
given torch-allocated scratch, at the tolerance the other parity tests use.
It also checks that an oversized request is refused with a clear error.  The
file name makes pytest collect it last; it passes alone in a fresh process as
well.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import attention as oatt

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def _inputs(Hq, Hkv, N, D, seed):
    g = torch.Generator().manual_seed(seed)
    mk = lambda *s: torch.randn(*s, generator=g).to(torch.float16).cuda()
    return mk(Hq, D), mk(Hkv, N, D), mk(Hkv, N, D)


def _with_caller_scratch(fqkv, q, K, V, S):
    Hq, D = q.shape
    Hkv, N, _ = K.shape
    mp = torch.empty(Hq, S, device="cuda")
    lp = torch.empty(Hq, S, device="cuda")
    op = torch.empty(Hq, S, D, device="cuda")
    out = torch.empty(Hq, D, dtype=torch.float16, device="cuda")
    rc = fqkv.native.lib().fqkv_gqa_sk_fast(q.data_ptr(), K.data_ptr(), V.data_ptr(), mp.data_ptr(), lp.data_ptr(),
                                            op.data_ptr(), out.data_ptr(), Hq, Hkv, N, D, S, 8, 8,
                                            torch.cuda.current_stream().cuda_stream)
    fqkv.native.check(rc, "fqkv_gqa_sk_fast")
    return out


def _static(fqkv, q, K, V, S):
    Hq, D = q.shape
    Hkv, N, _ = K.shape
    out = torch.empty(Hq, D, dtype=torch.float16, device="cuda")
    rc = fqkv.native.lib().fqkv_gqa_sk_fast_static_scratch(q.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr(),
                                                           Hq, Hkv, N, D, S, 8, 8,
                                                           torch.cuda.current_stream().cuda_stream)
    fqkv.native.check(rc, "fqkv_gqa_sk_fast_static_scratch")
    return out


def test_static_scratch_matches_caller_scratch_twice(fqkv):
    torch.cuda.set_device(0)
    for (Hq, Hkv, N, D, S, seed) in ((32, 8, 16384, 128, 64, 1), (32, 8, 3000, 64, 7, 2)):
        q, K, V = _inputs(Hq, Hkv, N, D, seed)
        got = _static(fqkv, q, K, V, S)
        ref = _with_caller_scratch(fqkv, q, K, V, S)
        torch.cuda.synchronize()
        torch.testing.assert_close(got.float(), ref.float(), atol=ATOL, rtol=RTOL)
        oracle = oatt.decode_attention_gqa(q.cpu().numpy()[None], K.cpu().numpy()[None], V.cpu().numpy()[None])[0]
        np.testing.assert_allclose(got.float().cpu().numpy().astype(np.float64), oracle, atol=ATOL, rtol=RTOL)


def test_static_scratch_rejects_oversized_request(fqkv):
    torch.cuda.set_device(0)
    q, K, V = _inputs(32, 8, 64, 128, 3)
    out = torch.empty(32, 128, dtype=torch.float16, device="cuda")
    rc = fqkv.native.lib().fqkv_gqa_sk_fast_static_scratch(q.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr(),
                                                           32, 8, 64, 128, 253, 8, 8, None)
    assert rc == fqkv.native.ERR_INVALID_ARGUMENT
    assert "static array" in fqkv.native.last_error()
    st = ctypes.c_int(-1)
    fqkv.native.check(fqkv.native.lib().fqkv_device_status(ctypes.byref(st), 0), "status")
    assert st.value == 0
