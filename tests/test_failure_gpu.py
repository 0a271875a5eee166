"""Failure detection without a GPU fault.

Every mbarrier wait in the decode kernels and the staged quantizers is bounded.
The test hook ``fqkv_debug_skip_loads`` makes the producer issue no tile loads, so the
consumers' waits for a tile run out after a short limit (a flag that nothing
sets).  The kernel must unwind on its own, record status 61 in the device
status word, and leave the CUDA context usable: the next normal launch
returns correct results.  Nothing faults, traps or hangs."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import quant as oq

pytestmark = pytest.mark.gpu


def _status(fqkv, clear=0):
    st = ctypes.c_int(-1)
    fqkv.native.check(fqkv.native.lib().fqkv_device_status(ctypes.byref(st), clear), "status")
    return st.value


@pytest.mark.parametrize("kind", ["gqa", "int8", "int4", "gqa_int8", "gqa_int8_cluster", "gqa_int8_cluster_long",
                                  "qpt", "quant_int4"])
def test_stalled_pipeline_times_out_and_context_survives(fqkv, kind):
    """A pipeline whose tiles never arrive: every bounded wait gives up, the kernel unwinds by itself
    (in the cluster-merge forms every thread still passes both cluster barriers), status 61 is
    recorded, and the context stays usable.  The "gqa" shape (N = 300) runs the fp16 cluster merge;
    the int8 cluster cases run its one-group (N = 300) and two-group (N = 4096) forms; "qpt" and
    "quant_int4" stall the staged quantizers' shared-memory ring."""
    lib = fqkv.native.lib()
    g = torch.Generator().manual_seed(5)
    B, Hq, Hkv, N, D = 2, 8, 2, 4096 if kind == "gqa_int8_cluster_long" else 300, 128
    q = torch.randn(B, Hq, D, generator=g).half().cuda()
    K = torch.randn(B, Hkv, N, D, generator=g).half().cuda()
    V = torch.randn(B, Hkv, N, D, generator=g).half().cuda()
    # quantized inputs are made before the hook is on (the quantizers honour it too)
    if kind == "int8":
        Kq, Ks = fqkv.qpt(K.view(B * Hkv, N, D))
        Vq, Vs = fqkv.qpt(V.view(B * Hkv, N, D))
    elif kind == "int4":
        Kp, Ks = fqkv.quant_int4_per_token(K.view(B * Hkv, N, D))
        Vp, Vs = fqkv.quant_int4_per_token(V.view(B * Hkv, N, D))
    elif kind.startswith("gqa_int8"):
        Kq, Ks = fqkv.qpt(K)
        Vq, Vs = fqkv.qpt(V)
    torch.cuda.synchronize()
    assert _status(fqkv, clear=1) == 0
    lib.fqkv_set_wait_timeout_ms(50)
    lib.fqkv_debug_skip_loads(1)
    try:
        if kind == "gqa":
            fqkv.decode_attn_gqa(q, K, V, 8)
        elif kind == "int8":
            fqkv.decode_attn_int8_mw(q[:, :Hkv].reshape(B * Hkv, D).contiguous(), Kq, Vq, Ks, Vs, 8)
        elif kind == "int4":  # tensor-core quantized kernel, one head per KV row
            fqkv.decode_attn_int4(q[:, :Hkv].reshape(B * Hkv, D).contiguous(), Kp, Vp, Ks, Vs, 8)
        elif kind == "qpt":
            fqkv.qpt(K)
        elif kind == "quant_int4":
            fqkv.quant_int4_per_token(K)
        else:  # tensor-core quantized kernel, several heads per KV row (forced: its cluster-merge form)
            if kind.startswith("gqa_int8_cluster"):
                fqkv.native.check(lib.fqkv_set_split_mode(fqkv.native.SPLIT_CLUSTER), "split mode")
            fqkv.decode_attn_gqa_int8(q, Kq, Vq, Ks, Vs)
        torch.cuda.synchronize()
    finally:
        lib.fqkv_debug_skip_loads(0)
        lib.fqkv_set_wait_timeout_ms(2000)
        lib.fqkv_set_split_mode(fqkv.native.SPLIT_AUTO)
    assert _status(fqkv, clear=1) == 61          # a consumer's wait for a tile ran out
    assert _status(fqkv) == 0
    out = fqkv.decode_attn_gqa(q, K, V, 8)        # the context is still healthy
    ref = oatt.decode_attention_gqa(q.cpu().numpy(), K.cpu().numpy(), V.cpu().numpy())
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=2e-3, rtol=1e-2)
    if kind in ("qpt", "quant_int4"):              # and the quantizer runs clean again
        c, s = fqkv.qpt(K)
        rc, rs = oq.quantize_int8_per_token(K.cpu().numpy())
        assert np.array_equal(c.cpu().numpy(), rc)
    assert _status(fqkv) == 0


def test_tensor_parallel_wait_times_out_on_missing_peer(fqkv):
    """The arrival wait of the fused tensor-parallel gather is bounded: counters
    that nothing advances (a peer that never sends) end the wait after the limit
    with status 64; the sequence still advances, later waits return at once while
    the status is set, and once the status is read and cleared a wait whose
    counts are in returns clean."""
    lib = fqkv.native.lib()
    counters = torch.zeros(2, dtype=torch.int64, device="cuda")     # this rank's slots for 2 ranks
    seq = torch.zeros(1, dtype=torch.int64, device="cuda")
    dev = counters.device
    assert _status(fqkv, clear=1) == 0
    lib.fqkv_set_wait_timeout_ms(50)
    try:
        fqkv.ops.tp_wait(counters.data_ptr(), 2, 3, seq.data_ptr(), dev)   # needs 3 arrivals per rank
        torch.cuda.synchronize()
    finally:
        lib.fqkv_set_wait_timeout_ms(2000)
    # a later wait while the status word still records the first timeout returns at once instead of
    # waiting out its own limit (a dead peer never catches up: every layer of every remaining step
    # would otherwise stall for the full limit before the host can read the status)
    lib.fqkv_set_wait_timeout_ms(3000)
    try:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(4):
            fqkv.ops.tp_wait(counters.data_ptr(), 2, 3, seq.data_ptr(), dev)
        e1.record()
        torch.cuda.synchronize()
    finally:
        lib.fqkv_set_wait_timeout_ms(2000)
    assert e0.elapsed_time(e1) < 500.0                                 # not 4 x 3 s
    assert int(seq.item()) == 5
    with pytest.raises(RuntimeError, match="tensor-parallel peer"):   # what GraphDecoder.generate raises
        fqkv.ops.check_device_status(dev, "decode step")
    assert _status(fqkv) == 0                                          # the check reset the word
    counters.fill_(18)                                                 # calls 1 .. 6 complete
    fqkv.ops.tp_wait(counters.data_ptr(), 2, 3, seq.data_ptr(), dev)
    torch.cuda.synchronize()
    assert _status(fqkv) == 0 and int(seq.item()) == 6
