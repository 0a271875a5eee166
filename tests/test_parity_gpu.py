"""GPU parity: every attention entry point against the CPU oracle.

Inputs are drawn on the CPU with ``torch.manual_seed`` (as the reference's
tests do), copied to the GPU, and the library's output is compared with the
float64 oracle at ``atol=2e-3, rtol=1e-2`` (the build's tolerance; the
reference's own tests use 2e-2 .. 6e-2).  Quantized paths are compared with
the oracle evaluated on the dequantised KV, codes coming from the library's
own quantizer (which ``test_quantizer_gpu.py`` pins bit-exact).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import quant as oq

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def _randn(*shape, seed=0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g, dtype=torch.float32).to(torch.float16)


def _close(out: torch.Tensor, ref: np.ndarray):
    got = out.float().cpu().numpy().astype(np.float64)
    np.testing.assert_allclose(got, ref, atol=ATOL, rtol=RTOL)


# ------------------------------------------------------------------ fp16 (K1)
# reference tests: (B,N,W) in {(1,1024,8),(8,2048,4),(256,4096,8)} at D=64
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("R,N,W", [(1, 1024, 8), (8, 2048, 4), (256, 4096, 8), (3, 1, 2), (2, 3, 4),
                                   (5, 100, 8), (4, 63, 8), (4, 64, 8), (4, 65, 8), (2, 16385, 8)])
def test_fp16_mw(fqkv, R, N, W, D):
    q, K, V = _randn(R, D, seed=1), _randn(R, N, D, seed=2), _randn(R, N, D, seed=3)
    out = fqkv.decode_attn_fp16_mw(q.cuda(), K.cuda(), V.cuda(), W)
    torch.cuda.synchronize()
    assert out.shape == (R, D) and out.dtype == torch.float16
    _close(out, oatt.decode_attention(q.numpy(), K.numpy(), V.numpy()))


def test_fp16_mw_full_cfg1(fqkv):
    """BASELINE config 1 at full size: B=8 x 32 heads, N=4096, D=128."""
    R, N, D = 256, 4096, 128
    q, K, V = _randn(R, D, seed=11), _randn(R, N, D, seed=12), _randn(R, N, D, seed=13)
    out = fqkv.decode_attn_fp16_mw(q.cuda(), K.cuda(), V.cuda(), 8)
    _close(out, oatt.decode_attention(q.numpy(), K.numpy(), V.numpy()))


# ------------------------------------------------------------------ int8 (K2)
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("R,N,W", [(1, 1024, 8), (8, 2048, 4), (3, 1, 2), (2, 3, 4), (5, 100, 8),
                                   (4, 64, 8), (4, 129, 8), (2, 5000, 8)])
def test_int8_mw(fqkv, R, N, W, D):
    q, K, V = _randn(R, D, seed=4), _randn(R, N, D, seed=5), _randn(R, N, D, seed=6)
    Kq, Ks = fqkv.qpt(K.cuda())
    Vq, Vs = fqkv.qpt(V.cuda())
    out = fqkv.decode_attn_int8_mw(q.cuda(), Kq, Vq, Ks, Vs, W)
    Kd = oq.dequantize_int8(Kq.cpu().numpy(), Ks.cpu().numpy())
    Vd = oq.dequantize_int8(Vq.cpu().numpy(), Vs.cpu().numpy())
    _close(out, oatt.decode_attention(q.numpy(), Kd, Vd))


# ------------------------------------------------------------------ int4 (K3)
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("R,N,W", [(1, 1024, 8), (8, 2048, 2), (256, 4096, 8), (4, 3, 4), (3, 1, 2),
                                   (5, 100, 8), (4, 257, 8)])
def test_int4(fqkv, R, N, W, D):
    q, K, V = _randn(R, D, seed=7), _randn(R, N, D, seed=8), _randn(R, N, D, seed=9)
    Kp, Ks = fqkv.quant_int4_per_token(K.cuda())
    Vp, Vs = fqkv.quant_int4_per_token(V.cuda())
    out = fqkv.decode_attn_int4(q.cuda(), Kp, Vp, Ks, Vs, W)
    Kd = oq.dequantize_int4(Kp.cpu().numpy(), Ks.cpu().numpy())
    Vd = oq.dequantize_int4(Vp.cpu().numpy(), Vs.cpu().numpy())
    _close(out, oatt.decode_attention(q.numpy(), Kd, Vd))


def test_quantized_inputs_with_zero_tokens(fqkv):
    """All-zero tokens quantize to scale 0 / codes 0 and contribute a zero key/value."""
    R, N, D = 2, 70, 128
    q, K, V = _randn(R, D, seed=20), _randn(R, N, D, seed=21), _randn(R, N, D, seed=22)
    K[:, 5] = 0
    V[:, 5] = 0
    V[:, 66] = 0
    for quant, dq, op in ((fqkv.qpt, oq.dequantize_int8, fqkv.decode_attn_int8_mw),
                          (fqkv.quant_int4_per_token, oq.dequantize_int4, fqkv.decode_attn_int4)):
        Kc, Ks = quant(K.cuda())
        Vc, Vs = quant(V.cuda())
        assert float(Ks[0, 5]) == 0.0
        out = op(q.cuda(), Kc, Vc, Ks, Vs, 8)
        ref = oatt.decode_attention(q.numpy(), dq(Kc.cpu().numpy(), Ks.cpu().numpy()),
                                    dq(Vc.cpu().numpy(), Vs.cpu().numpy()))
        _close(out, ref)


# ------------------------------------------------------------------ GQA (K4)
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("B,Hq,Hkv,N", [(1, 32, 8, 1024), (16, 32, 8, 4096), (2, 32, 8, 37), (3, 32, 8, 1),
                                        (2, 8, 8, 300), (2, 64, 8, 200), (1, 32, 2, 500), (2, 12, 4, 129),
                                        (1, 32, 8, 16384)])
def test_gqa(fqkv, B, Hq, Hkv, N, D):
    q, K, V = _randn(B, Hq, D, seed=30), _randn(B, Hkv, N, D, seed=31), _randn(B, Hkv, N, D, seed=32)
    out = fqkv.decode_attn_gqa(q.cuda(), K.cuda(), V.cuda(), 8)
    assert out.shape == (B, Hq, D)
    _close(out, oatt.decode_attention_gqa(q.numpy(), K.numpy(), V.numpy()))


def test_gqa_bench_shape_sampled_rows(fqkv):
    """The bench workload (B=64, Hq=32, Hkv=8, N=16384, D=128), checked on sampled sequences."""
    B, Hq, Hkv, N, D = 64, 32, 8, 16384, 128
    gen = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(B, Hq, D, device="cuda", generator=gen, dtype=torch.float16)
    K = torch.randn(B, Hkv, N, D, device="cuda", generator=gen, dtype=torch.float16)
    V = torch.randn(B, Hkv, N, D, device="cuda", generator=gen, dtype=torch.float16)
    out = fqkv.decode_attn_gqa(q, K, V, 8)
    for b in (0, 17, 63):
        ref = oatt.decode_attention_gqa(q[b:b + 1].cpu().numpy(), K[b:b + 1].cpu().numpy(),
                                        V[b:b + 1].cpu().numpy())
        _close(out[b:b + 1], ref)


# ------------------------------------------------------------------ split-K (K5-K7)
# the reference's six cases (tests/test_kernels.py:59) plus larger S / N
@pytest.mark.parametrize("N,D,S,W,CW", [(1024, 64, 8, 8, 4), (4096, 128, 16, 8, 4), (16384, 64, 64, 8, 8),
                                        (3, 128, 8, 4, 4), (1, 64, 4, 2, 4), (100, 64, 7, 4, 4),
                                        (16384, 128, 64, 8, 8), (65536, 128, 128, 8, 8), (777, 128, 1, 8, 4),
                                        (8192, 64, 64, 8, 8)])
def test_gqa_sk_fast(fqkv, N, D, S, W, CW):
    Hq, Hkv = 32, 8
    q, K, V = _randn(Hq, D, seed=40), _randn(Hkv, N, D, seed=41), _randn(Hkv, N, D, seed=42)
    dev = "cuda"
    mp = torch.empty(Hq, S, dtype=torch.float32, device=dev)
    lp = torch.empty(Hq, S, dtype=torch.float32, device=dev)
    op = torch.empty(Hq, S, D, dtype=torch.float32, device=dev)
    out = torch.empty(Hq, D, dtype=torch.float16, device=dev)
    fqkv.gqa_sk_fast(q.cuda(), K.cuda(), V.cuda(), mp, lp, op, out, S, W, CW)
    _close(out, oatt.decode_attention_gqa(q.numpy()[None], K.numpy()[None], V.numpy()[None])[0])


# ------------------------------------------------------------------ properties
def test_split_count_does_not_change_the_result(fqkv):
    """Same op with no workspace (one split) and with the preferred split-K plan (partials +
    combine: at D = 64 batch 1 past N = 8192 does not use the cluster merge)."""
    B, Hq, Hkv, N, D = 1, 32, 8, 16384, 64
    q, K, V = (_randn(B, Hq, D, seed=50).cuda(), _randn(B, Hkv, N, D, seed=51).cuda(),
               _randn(B, Hkv, N, D, seed=52).cuda())
    lib = fqkv.native.lib()
    out1 = torch.empty(B, Hq, D, dtype=torch.float16, device="cuda")
    rc = lib.fqkv_decode_attn_gqa(q.data_ptr(), K.data_ptr(), V.data_ptr(), out1.data_ptr(), B, Hq, Hkv, N, D, 8,
                                  None, 0, torch.cuda.current_stream().cuda_stream)
    fqkv.native.check(rc, "gqa")
    nb = fqkv.workspace_bytes("fp16", B, Hq, Hkv, N, D)
    assert nb > 0
    ws = torch.empty(nb, dtype=torch.uint8, device="cuda")
    out2 = torch.empty_like(out1)
    rc = lib.fqkv_decode_attn_gqa(q.data_ptr(), K.data_ptr(), V.data_ptr(), out2.data_ptr(), B, Hq, Hkv, N, D, 8,
                                  ws.data_ptr(), nb, torch.cuda.current_stream().cuda_stream)
    fqkv.native.check(rc, "gqa")
    torch.testing.assert_close(out1.float(), out2.float(), atol=1e-3, rtol=1e-3)


def test_cuda_graph_capture_and_side_stream(fqkv):
    B, Hq, Hkv, N, D = 2, 32, 8, 4096, 128
    q, K, V = (_randn(B, Hq, D, seed=60).cuda(), _randn(B, Hkv, N, D, seed=61).cuda(),
               _randn(B, Hkv, N, D, seed=62).cuda())
    ref = fqkv.decode_attn_gqa(q, K, V, 8)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        side = fqkv.decode_attn_gqa(q, K, V, 8)
    torch.cuda.current_stream().wait_stream(s)
    torch.testing.assert_close(side, ref, atol=0, rtol=0)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        cap = fqkv.decode_attn_gqa(q, K, V, 8)
    g.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(cap, ref, atol=0, rtol=0)


def test_split_launches_on_two_streams_at_once(fqkv):
    """Split launches (partial kernel + combine) in flight on two streams at once, each with its own workspace
    (D = 64: batch 1 past N = 8192 splits into partials + combine there)."""
    B, Hq, Hkv, N, D = 1, 32, 8, 16384, 64
    assert fqkv.workspace_bytes("fp16", B, Hq, Hkv, N, D) > 0
    inputs = [(_randn(B, Hq, D, seed=100 + i).cuda(), _randn(B, Hkv, N, D, seed=110 + i).cuda(),
               _randn(B, Hkv, N, D, seed=120 + i).cuda()) for i in range(2)]
    refs = [fqkv.decode_attn_gqa(*x, 8) for x in inputs]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    for st in streams:
        st.wait_stream(torch.cuda.current_stream())
    outs = [[], []]
    for _ in range(20):
        for i, st in enumerate(streams):
            with torch.cuda.stream(st):
                outs[i].append(fqkv.decode_attn_gqa(*inputs[i], 8))
    for st in streams:
        torch.cuda.current_stream().wait_stream(st)
    torch.cuda.synchronize()
    for i in range(2):
        for o in outs[i]:
            assert torch.equal(o, refs[i])


def test_device_status_clean_after_suite(fqkv):
    import ctypes
    st = ctypes.c_int(-1)
    fqkv.native.check(fqkv.native.lib().fqkv_device_status(ctypes.byref(st), 0), "status")
    assert st.value == 0


# ------------------------------------------------------------------ KV-cache entry (model decode step)
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("B,Hq,Hkv,max_len,n", [(1, 32, 8, 640, 513), (4, 32, 8, 300, 1), (2, 16, 2, 5000, 4097),
                                                (64, 32, 8, 640, 600)])
def test_gqa_kvcache_host_and_device_length(fqkv, B, Hq, Hkv, max_len, n, D):
    q = _randn(B, Hq, D, seed=70).cuda()
    K = torch.zeros(B, Hkv, max_len, D, dtype=torch.float16, device="cuda")
    V = torch.zeros_like(K)
    K[:, :, :n] = _randn(B, Hkv, n, D, seed=71).cuda()
    V[:, :, :n] = _randn(B, Hkv, n, D, seed=72).cuda()
    ref = oatt.decode_attention_gqa(q.cpu().numpy(), K[:, :, :n].cpu().numpy(), V[:, :, :n].cpu().numpy())
    _close(fqkv.decode_attn_gqa_kvcache(q, K, V, n), ref)
    n_dev = torch.tensor([n], dtype=torch.int32, device="cuda")
    _close(fqkv.decode_attn_gqa_kvcache(q, K, V, n_dev), ref)


def test_gqa_kvcache_graph_follows_device_length(fqkv):
    B, Hq, Hkv, max_len, D = 2, 32, 8, 1024, 64
    q = _randn(B, Hq, D, seed=80).cuda()
    K = _randn(B, Hkv, max_len, D, seed=81).cuda()
    V = _randn(B, Hkv, max_len, D, seed=82).cuda()
    n_dev = torch.tensor([100], dtype=torch.int32, device="cuda")
    out = torch.empty(B, Hq, D, dtype=torch.float16, device="cuda")
    ws = torch.empty(max(fqkv.workspace_bytes("fp16", B, Hq, Hkv, max_len, D), 1), dtype=torch.uint8, device="cuda")
    fqkv.decode_attn_gqa_kvcache(q, K, V, n_dev, out=out, workspace=ws)   # first call: device set-up
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fqkv.decode_attn_gqa_kvcache(q, K, V, n_dev, out=out, workspace=ws)
    for n in (100, 101, 513, 1024, 7):
        n_dev.fill_(n)
        g.replay()
        torch.cuda.synchronize()
        ref = oatt.decode_attention_gqa(q.cpu().numpy(), K[:, :, :n].cpu().numpy(), V[:, :, :n].cpu().numpy())
        _close(out, ref)


# ------------------------------------------------------------------ int8-KV GQA (model int8 cache)
def _int8_gqa_ref(q, Kf, Vf, n=None):
    """Oracle on the reference quantizer's dequantised int8 KV (first n keys)."""
    Kc, Ks = oq.quantize_int8_per_token(Kf)
    Vc, Vs = oq.quantize_int8_per_token(Vf)
    Kd, Vd = oq.dequantize_int8(Kc, Ks), oq.dequantize_int8(Vc, Vs)
    if n is not None:
        Kd, Vd = Kd[:, :, :n], Vd[:, :, :n]
    return oatt.decode_attention_gqa(q, Kd, Vd)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("B,Hq,Hkv,N", [(1, 32, 8, 1024), (4, 32, 8, 513), (2, 64, 8, 77), (3, 8, 2, 1),
                                        (1, 32, 8, 16384), (2, 12, 4, 300), (1, 128, 8, 200), (2, 16, 8, 130),
                                        (1, 40, 8, 63)])
def test_gqa_int8(fqkv, B, Hq, Hkv, N, D):
    q, K, V = _randn(B, Hq, D, seed=90), _randn(B, Hkv, N, D, seed=91), _randn(B, Hkv, N, D, seed=92)
    Kq, Ks = fqkv.qpt(K.cuda())
    Vq, Vs = fqkv.qpt(V.cuda())
    out = fqkv.decode_attn_gqa_int8(q.cuda(), Kq, Vq, Ks, Vs)
    _close(out, _int8_gqa_ref(q.numpy(), K.numpy(), V.numpy()))


@pytest.mark.parametrize("int4", [False, True])
def test_quantize_into_cache_bit_exact(fqkv, int4):
    G, T, D, cap = 6, 37, 128, 100
    X = _randn(G, T, D, seed=93)
    codes = torch.zeros(G, cap, D // 2 if int4 else D, dtype=torch.uint8 if int4 else torch.int8, device="cuda")
    scales = torch.zeros(G, cap, dtype=torch.float16, device="cuda")
    fqkv.quantize_into_cache(X.cuda(), codes, scales, 10, int4=int4)
    rc, rs = (oq.quantize_int4_per_token if int4 else oq.quantize_int8_per_token)(X.numpy())
    assert np.array_equal(codes[:, 10:10 + T].cpu().numpy(), rc)
    assert np.array_equal(scales[:, 10:10 + T].cpu().numpy().view(np.uint16), rs.view(np.uint16))
    assert not codes[:, :10].any() and not codes[:, 10 + T:].any()
    # device position, one token per group, graph-style append; a position past cap writes nothing
    x1 = _randn(G, 1, D, seed=94).cuda()
    pos = torch.tensor([99], dtype=torch.int32, device="cuda")
    fqkv.quantize_into_cache(x1, codes, scales, pos, int4=int4)
    r1c, r1s = (oq.quantize_int4_per_token if int4 else oq.quantize_int8_per_token)(x1.cpu().numpy())
    assert np.array_equal(codes[:, 99:100].cpu().numpy(), r1c)
    before = codes.clone()
    pos.fill_(100)
    fqkv.quantize_into_cache(x1, codes, scales, pos, int4=int4)
    torch.cuda.synchronize()
    assert torch.equal(before, codes)


@pytest.mark.parametrize("B,Hq,Hkv,max_len,n,D", [(1, 32, 8, 640, 513, 64), (8, 32, 8, 640, 600, 64),
                                                  (2, 32, 8, 4096, 4000, 128)])
def test_gqa_int8_kvcache_append_and_device_length(fqkv, B, Hq, Hkv, max_len, n, D):
    q = _randn(B, Hq, D, seed=95)
    Kf, Vf = _randn(B, Hkv, n, D, seed=96), _randn(B, Hkv, n, D, seed=97)
    Kq = torch.zeros(B, Hkv, max_len, D, dtype=torch.int8, device="cuda")
    Vq = torch.zeros_like(Kq)
    Ks = torch.zeros(B, Hkv, max_len, dtype=torch.float16, device="cuda")
    Vs = torch.zeros_like(Ks)
    fqkv.quantize_into_cache(Kf[:, :, :n - 1].contiguous().cuda(), Kq, Ks, 0)   # prefill
    fqkv.quantize_into_cache(Vf[:, :, :n - 1].contiguous().cuda(), Vq, Vs, 0)
    pos = torch.tensor([n - 1], dtype=torch.int32, device="cuda")                # one appended token
    fqkv.quantize_into_cache(Kf[:, :, n - 1:].contiguous().cuda(), Kq, Ks, pos)
    fqkv.quantize_into_cache(Vf[:, :, n - 1:].contiguous().cuda(), Vq, Vs, pos)
    ref = _int8_gqa_ref(q.numpy(), Kf.numpy(), Vf.numpy())
    _close(fqkv.decode_attn_gqa_int8_kvcache(q.cuda(), Kq, Vq, Ks, Vs, n), ref)
    n_dev = torch.tensor([n], dtype=torch.int32, device="cuda")
    _close(fqkv.decode_attn_gqa_int8_kvcache(q.cuda(), Kq, Vq, Ks, Vs, n_dev), ref)


@pytest.mark.parametrize("kv", ["fp16", "int8"])
@pytest.mark.parametrize("B,n,D", [(8, 513, 64), (2, 4097, 128), (16, 40, 64)])
def test_kvcache_bf16_output(fqkv, kv, B, n, D):
    """bf16 output (for a bf16 model's output projection): the oracle within the fp16 tolerance plus one
    bf16 rounding, and the fp16 output's value within one bf16 rounding of each other (split and unsplit)."""
    Hq, Hkv, max_len = 32, 8, n + 100
    q = _randn(B, Hq, D, seed=130)
    Kf, Vf = _randn(B, Hkv, n, D, seed=131), _randn(B, Hkv, n, D, seed=132)
    n_dev = torch.tensor([n], dtype=torch.int32, device="cuda")
    if kv == "fp16":
        K = torch.zeros(B, Hkv, max_len, D, dtype=torch.float16, device="cuda")
        V = torch.zeros_like(K)
        K[:, :, :n], V[:, :, :n] = Kf.cuda(), Vf.cuda()
        ref = oatt.decode_attention_gqa(q.numpy(), Kf.numpy(), Vf.numpy())
        call = lambda out, ws: fqkv.decode_attn_gqa_kvcache(q.cuda(), K, V, n_dev, out=out, workspace=ws)
    else:
        Kq = torch.zeros(B, Hkv, max_len, D, dtype=torch.int8, device="cuda")
        Vq = torch.zeros_like(Kq)
        Ks = torch.zeros(B, Hkv, max_len, dtype=torch.float16, device="cuda")
        Vs = torch.zeros_like(Ks)
        fqkv.quantize_into_cache(Kf.cuda(), Kq, Ks, 0)
        fqkv.quantize_into_cache(Vf.cuda(), Vq, Vs, 0)
        ref = _int8_gqa_ref(q.numpy(), Kf.numpy(), Vf.numpy())
        call = lambda out, ws: fqkv.decode_attn_gqa_int8_kvcache(q.cuda(), Kq, Vq, Ks, Vs, n_dev, out=out,
                                                                  workspace=ws)
    nb = fqkv.workspace_bytes(kv, B, Hq, Hkv, max_len, D)
    for ws in (torch.empty(max(nb, 16), dtype=torch.uint8, device="cuda"), torch.empty(0, dtype=torch.uint8,
                                                                                          device="cuda")):
        o16 = call(torch.empty(B, Hq, D, dtype=torch.float16, device="cuda"), ws)
        ob = call(torch.empty(B, Hq, D, dtype=torch.bfloat16, device="cuda"), ws)
        assert ob.dtype == torch.bfloat16
        got = ob.float().cpu().numpy().astype(np.float64)
        bf_ulp = 2.0 ** -8 * np.abs(ref)
        np.testing.assert_allclose(got, ref, atol=ATOL, rtol=RTOL + 2.0 ** -8)
        diff = (ob.float() - o16.float()).abs()
        assert (diff <= 2.0 ** -8 * o16.float().abs() + 2.0 ** -11 * o16.float().abs() + 1e-6).all()


def test_gqa_int8_extreme_q_and_scales(fqkv):
    """q with one huge element per head (fixed-point q planes lose the small ones
    only below the tolerance), all-zero tokens (scale 0), a zero q head."""
    B, Hq, Hkv, N, D = 2, 16, 4, 300, 128
    q = _randn(B, Hq, D, seed=98)
    q[:, :, 5] = 60.0
    q[1, 3] = 0.0
    K, V = _randn(B, Hkv, N, D, seed=99), _randn(B, Hkv, N, D, seed=100)
    K[:, :, 7] = 0.0
    V[:, :, 11] = 0.0
    V[0, 1, 13] *= 100.0
    Kq, Ks = fqkv.qpt(K.cuda())
    Vq, Vs = fqkv.qpt(V.cuda())
    out = fqkv.decode_attn_gqa_int8(q.cuda(), Kq, Vq, Ks, Vs)
    _close(out, _int8_gqa_ref(q.numpy(), K.numpy(), V.numpy()))


@pytest.mark.parametrize("D", [64, 128])
def test_int4_extreme_q_and_scales(fqkv, D):
    """int4 with a dominant q element (the fixed-point q planes and the +8 nibble
    bias correction at their extremes), a zero q row, zero tokens and a token
    with a 100x larger scale."""
    R, N = 6, 700
    q = _randn(R, D, seed=101)
    q[:, 3] = -60.0
    q[2] = 0.0
    q[4] *= 30.0
    K, V = _randn(R, N, D, seed=102), _randn(R, N, D, seed=103)
    K[:, 10] = 0.0
    V[:, 20] = 0.0
    V[1, 33] *= 100.0
    K[3, 44] *= 100.0
    Kp, Ks = fqkv.quant_int4_per_token(K.cuda())
    Vp, Vs = fqkv.quant_int4_per_token(V.cuda())
    out = fqkv.decode_attn_int4(q.cuda(), Kp, Vp, Ks, Vs, 8)
    Kd = oq.dequantize_int4(Kp.cpu().numpy(), Ks.cpu().numpy())
    Vd = oq.dequantize_int4(Vp.cpu().numpy(), Vs.cpu().numpy())
    _close(out, oatt.decode_attention(q.numpy(), Kd, Vd))


def test_int4_frames_under_moving_maximum_and_scales(fqkv):
    """int4 at D=128 with units long enough to span many tiles (R=288 runs
    unsplit, 32 tiles per unit): scores with a dominant q element move the
    running maximum by more than 2^3 many times per unit, and V scales spread
    over five decades (plus zero tokens) move the fixed-point range of P*V, so
    the kernel's integer accumulators are flushed and rescaled mid-unit over
    and over.  Sampled rows against the oracle."""
    R, N, D = 288, 4096, 128
    g = torch.Generator().manual_seed(140)
    q = torch.randn(R, D, generator=g)
    q[:, 0] = 20.0
    K = torch.randn(R, N, D, generator=g) * 0.3
    K[:, :, 0] = torch.randn(R, N, generator=g) * 3.0
    V = torch.randn(R, N, D, generator=g) * torch.pow(10.0, torch.rand(R, N, 1, generator=g) * 5.0 - 3.0)
    K[:, 200] = 0.0
    V[:, 100] = 0.0
    q, K, V = q.half(), K.half(), V.half()
    Kp, Ks = fqkv.quant_int4_per_token(K.cuda())
    Vp, Vs = fqkv.quant_int4_per_token(V.cuda())
    out = fqkv.decode_attn_int4(q.cuda(), Kp, Vp, Ks, Vs, 8)
    rows = [0, 1, 2, 77, 143, 200, 255, 287]
    Kd = oq.dequantize_int4(Kp[rows].cpu().numpy(), Ks[rows].cpu().numpy())
    Vd = oq.dequantize_int4(Vp[rows].cpu().numpy(), Vs[rows].cpu().numpy())
    _close(out[rows], oatt.decode_attention(q[rows].numpy(), Kd, Vd))


# ------------------------------------------------------------------ unwritten KV-cache tails
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("B,Hq,Hkv,max_len,n", [(2, 32, 8, 200, 100), (1, 32, 8, 4096, 3001), (3, 8, 8, 300, 129),
                                                (64, 32, 8, 640, 513)])
def test_kvcache_tail_of_nan_and_inf_is_ignored(fqkv, B, Hq, Hkv, max_len, n, D):
    """A cache allocated with torch.empty and written only up to n: positions [n, max_len) hold NaN
    and inf (fp16 K/V; int8 scales), and are read by the last tile of each unit.  The outputs must
    equal the oracle on the first n positions (host and device length, split and unsplit plans)."""
    q = _randn(B, Hq, D, seed=150)
    Kf, Vf = _randn(B, Hkv, n, D, seed=151), _randn(B, Hkv, n, D, seed=152)
    K = torch.empty(B, Hkv, max_len, D, dtype=torch.float16, device="cuda")
    V = torch.empty_like(K)
    K[:, :, n:] = float("nan")
    V[:, :, n:] = float("inf")
    V[:, :, n + 1::3] = float("nan")
    V[:, :, n + 2::3] = float("-inf")
    K[:, :, :n], V[:, :, :n] = Kf.cuda(), Vf.cuda()
    n_dev = torch.tensor([n], dtype=torch.int32, device="cuda")
    ref = oatt.decode_attention_gqa(q.numpy(), Kf.numpy(), Vf.numpy())
    for seq_len in (n, n_dev):
        for ws in (None, torch.empty(0, dtype=torch.uint8, device="cuda")):   # preferred plan, unsplit
            out = fqkv.decode_attn_gqa_kvcache(q.cuda(), K, V, seq_len, workspace=ws)
            assert torch.isfinite(out).all()
            _close(out, ref)
    # int8 cache: garbage codes past n and NaN / inf scales
    Kq = torch.randint(-128, 128, (B, Hkv, max_len, D), dtype=torch.int8, device="cuda")
    Vq = torch.randint(-128, 128, (B, Hkv, max_len, D), dtype=torch.int8, device="cuda")
    Ks = torch.full((B, Hkv, max_len), float("nan"), dtype=torch.float16, device="cuda")
    Vs = torch.full((B, Hkv, max_len), float("inf"), dtype=torch.float16, device="cuda")
    Vs[:, :, n + 1::2] = float("nan")
    fqkv.quantize_into_cache(Kf.cuda(), Kq, Ks, 0)
    fqkv.quantize_into_cache(Vf.cuda(), Vq, Vs, 0)
    ref8 = _int8_gqa_ref(q.numpy(), Kf.numpy(), Vf.numpy())
    for seq_len in (n, n_dev):
        for ws in (None, torch.empty(0, dtype=torch.uint8, device="cuda")):
            out = fqkv.decode_attn_gqa_int8_kvcache(q.cuda(), Kq, Vq, Ks, Vs, seq_len, workspace=ws)
            assert torch.isfinite(out).all()
            _close(out, ref8)


# ------------------------------------------------------------------ split merge: cluster (DSMEM) vs combine kernel
@pytest.fixture
def split_mode(fqkv):
    lib = fqkv.native.lib()

    def set_mode(m):
        fqkv.native.check(lib.fqkv_set_split_mode(m), "set_split_mode")
    yield set_mode
    set_mode(fqkv.native.SPLIT_AUTO)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("B,Hq,Hkv,N", [(1, 32, 8, 16384), (1, 32, 8, 65536), (1, 32, 8, 1000), (1, 32, 8, 65),
                                        (2, 32, 8, 4097), (1, 8, 1, 3000), (1, 64, 4, 2048), (3, 12, 4, 777),
                                        (1, 32, 2, 9000)])
def test_split_merge_modes_agree_with_oracle(fqkv, split_mode, B, Hq, Hkv, N, D):
    """The same split plan merged in one launch through a thread-block cluster's distributed shared
    memory, and by the partials + combine kernel pair: both against the oracle, and each other."""
    q, K, V = (_randn(B, Hq, D, seed=160).cuda(), _randn(B, Hkv, N, D, seed=161).cuda(),
               _randn(B, Hkv, N, D, seed=162).cuda())
    ref = oatt.decode_attention_gqa(q.cpu().numpy(), K.cpu().numpy(), V.cpu().numpy())
    outs = {}
    for mode in (fqkv.native.SPLIT_CLUSTER, fqkv.native.SPLIT_COMBINE, fqkv.native.SPLIT_AUTO):
        split_mode(mode)
        outs[mode] = fqkv.decode_attn_gqa(q, K, V, 8)
        _close(outs[mode], ref)
    torch.testing.assert_close(outs[fqkv.native.SPLIT_CLUSTER].float(), outs[fqkv.native.SPLIT_COMBINE].float(),
                               atol=1e-3, rtol=1e-3)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("B,Hq,Hkv,N", [(1, 32, 8, 16384), (1, 32, 8, 1000), (1, 32, 8, 65), (2, 32, 8, 4097),
                                        (1, 8, 1, 3000), (1, 64, 4, 2048), (3, 12, 4, 777), (4, 32, 8, 640)])
def test_int8_gqa_split_merge_modes_agree_with_oracle(fqkv, split_mode, B, Hq, Hkv, N, D):
    """int8 GQA on the tensor-core kernel: a split plan merged in one launch through a thread-block
    cluster's distributed shared memory, and by the partials + combine kernel pair -- both against
    the oracle on the dequantised cache, and each other."""
    q = _randn(B, Hq, D, seed=190).cuda()
    Kq, Ks = fqkv.qpt(_randn(B, Hkv, N, D, seed=191).cuda())
    Vq, Vs = fqkv.qpt(_randn(B, Hkv, N, D, seed=192).cuda())
    ref = oatt.decode_attention_gqa(q.cpu().numpy(), oq.dequantize_int8(Kq.cpu().numpy(), Ks.cpu().numpy()),
                                    oq.dequantize_int8(Vq.cpu().numpy(), Vs.cpu().numpy()))
    outs = {}
    for mode in (fqkv.native.SPLIT_CLUSTER, fqkv.native.SPLIT_COMBINE, fqkv.native.SPLIT_AUTO):
        split_mode(mode)
        outs[mode] = fqkv.decode_attn_gqa_int8(q, Kq, Vq, Ks, Vs)
        _close(outs[mode], ref)
    torch.testing.assert_close(outs[fqkv.native.SPLIT_CLUSTER].float(), outs[fqkv.native.SPLIT_COMBINE].float(),
                               atol=1e-3, rtol=1e-3)


@pytest.mark.parametrize("D", [64, 128])
def test_int8_gqa_cluster_merge_kvcache_in_graph(fqkv, split_mode, D):
    """The int8 GQA cluster merge over a device-length cache whose tail holds garbage codes and NaN /
    inf scales, inside a CUDA graph replayed as the cache grows."""
    split_mode(fqkv.native.SPLIT_CLUSTER)
    B, Hq, Hkv, max_len = 1, 32, 8, 8192
    q = _randn(B, Hq, D, seed=193).cuda()
    Kq = torch.randint(-127, 128, (B, Hkv, max_len, D), dtype=torch.int8, device="cuda")
    Vq = torch.randint(-127, 128, (B, Hkv, max_len, D), dtype=torch.int8, device="cuda")
    Ks = torch.full((B, Hkv, max_len), float("nan"), dtype=torch.float16, device="cuda")
    Vs = torch.full_like(Ks, float("inf"))
    k8, ks = fqkv.qpt(_randn(B, Hkv, 6000, D, seed=194).cuda())
    v8, vs = fqkv.qpt(_randn(B, Hkv, 6000, D, seed=195).cuda())
    Kq[:, :, :6000], Ks[:, :, :6000], Vq[:, :, :6000], Vs[:, :, :6000] = k8, ks, v8, vs
    n_dev = torch.tensor([100], dtype=torch.int32, device="cuda")
    o = torch.empty(B, Hq, D, dtype=torch.float16, device="cuda")
    fqkv.decode_attn_gqa_int8_kvcache(q, Kq, Vq, Ks, Vs, n_dev, out=o)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fqkv.decode_attn_gqa_int8_kvcache(q, Kq, Vq, Ks, Vs, n_dev, out=o)
    for n in (100, 64, 1, 4097, 6000, 5999):
        n_dev.fill_(n)
        g.replay()
        torch.cuda.synchronize()
        ref = oatt.decode_attention_gqa(q.cpu().numpy(),
                                        oq.dequantize_int8(Kq[:, :, :n].cpu().numpy(), Ks[:, :, :n].cpu().numpy()),
                                        oq.dequantize_int8(Vq[:, :, :n].cpu().numpy(), Vs[:, :, :n].cpu().numpy()))
        assert torch.isfinite(o).all()
        _close(o, ref)


@pytest.mark.parametrize("D", [64, 128])
def test_cluster_merge_sk_fast_and_kvcache(fqkv, split_mode, D):
    """gqa_sk_fast (batch 1) and a device-length KV cache with a NaN tail, in cluster mode, inside a
    CUDA graph replayed as the cache grows."""
    split_mode(fqkv.native.SPLIT_CLUSTER)
    Hq, Hkv, N = 32, 8, 16384
    q, K, V = _randn(Hq, D, seed=170), _randn(Hkv, N, D, seed=171), _randn(Hkv, N, D, seed=172)
    S = 64
    mp = torch.empty(Hq, S, device="cuda")
    lp = torch.empty(Hq, S, device="cuda")
    op = torch.empty(Hq, S, D, device="cuda")
    out = torch.empty(Hq, D, dtype=torch.float16, device="cuda")
    fqkv.gqa_sk_fast(q.cuda(), K.cuda(), V.cuda(), mp, lp, op, out, S, 8, 8)
    _close(out, oatt.decode_attention_gqa(q.numpy()[None], K.numpy()[None], V.numpy()[None])[0])

    B, max_len = 1, 8192
    qc = _randn(B, Hq, D, seed=173).cuda()
    Kc = torch.full((B, Hkv, max_len, D), float("nan"), dtype=torch.float16, device="cuda")
    Vc = torch.full_like(Kc, float("inf"))
    Kc[:, :, :6000] = _randn(B, Hkv, 6000, D, seed=174).cuda()
    Vc[:, :, :6000] = _randn(B, Hkv, 6000, D, seed=175).cuda()
    n_dev = torch.tensor([100], dtype=torch.int32, device="cuda")
    o = torch.empty(B, Hq, D, dtype=torch.float16, device="cuda")
    ws = torch.empty(max(fqkv.workspace_bytes("fp16", B, Hq, Hkv, max_len, D), 16), dtype=torch.uint8, device="cuda")
    fqkv.decode_attn_gqa_kvcache(qc, Kc, Vc, n_dev, out=o, workspace=ws)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fqkv.decode_attn_gqa_kvcache(qc, Kc, Vc, n_dev, out=o, workspace=ws)
    for n in (100, 64, 1, 4097, 6000, 5999):
        n_dev.fill_(n)
        g.replay()
        torch.cuda.synchronize()
        ref = oatt.decode_attention_gqa(qc.cpu().numpy(), Kc[:, :, :n].cpu().numpy(), Vc[:, :, :n].cpu().numpy())
        assert torch.isfinite(o).all()
        _close(o, ref)


def test_split_plans_pick_the_cluster_merge_where_it_fits(fqkv):
    """Automatic split merging: a D = 128 split plan merges through a thread-block cluster (one
    launch, no workspace) when its whole grid of clusters is resident at once -- e.g. B=4, Hkv=8
    (32 clusters of 4), or through smaller clusters when the grid-filling size is not all resident
    (batch 1 with 8 KV heads: 8 clusters of 16 do not fit on B200, 8 of 10 do) up to N = 32K --
    and otherwise through partials + the combine kernel.  The batch-64 bench shape stays unsplit."""
    import ctypes
    lib = fqkv.native.lib()
    info = (ctypes.c_int32 * 33)()
    fqkv.native.check(lib.fqkv_device_info(info, 33), "device_info")
    max_clusters_128 = {c: info[3 + c - 2] for c in range(2, 17)}
    out = (ctypes.c_int32 * 5)()
    fqkv.native.check(lib.fqkv_decode_plan(0, 4, 32, 8, 16384, 128, 0, out), "plan")
    splits, cluster, grid, chunk, kernel = list(out)
    assert splits > 1 and cluster == splits and grid == 32 * splits and kernel == 0, list(out)
    assert fqkv.workspace_bytes("fp16", 4, 32, 8, 16384, 128) == 0
    # batch 1 (8 units): the largest cluster size whose 8 clusters are all resident (B200: 10 of
    # 16), taken automatically up to N = 32K; longer contexts keep partials + combine
    sm = info[0]
    fits = [c for c in range(2, min(16, sm // 8) + 1) if max_clusters_128[c] >= 8 and 2 * 8 * c >= sm]
    fqkv.native.check(lib.fqkv_decode_plan(0, 1, 32, 8, 16384, 128, 1 << 30, out), "plan")
    if fits:
        assert out[1] == out[0] == max(fits), (list(out), fits)
        assert fqkv.workspace_bytes("fp16", 1, 32, 8, 16384, 128) == 0
    else:
        assert out[0] > 1 and out[1] == 0, list(out)
    fqkv.native.check(lib.fqkv_decode_plan(0, 1, 32, 8, 65536, 128, 1 << 30, out), "plan")
    assert out[0] > 1 and out[1] == 0, list(out)
    assert fqkv.workspace_bytes("fp16", 1, 32, 8, 65536, 128) > 0
    fqkv.native.check(lib.fqkv_decode_plan(0, 64, 32, 8, 16384, 128, 0, out), "plan")
    assert out[0] == 1 and out[1] == 0
    # short contexts at D = 64 (the decode step of a Llama-1B-architecture model: N = 640) merge in a
    # cluster too, even where the split search alone would not split (batch 8, N = 512); long ones
    # keep partials + combine
    max_clusters_64 = {c: info[18 + c - 2] for c in range(2, 17)}
    for B, N in ((1, 640), (4, 640), (8, 512)):
        units = B * 8
        fits64 = [c for c in range(2, min(16, N // 64, sm // units) + 1) if max_clusters_64[c] >= units]
        fqkv.native.check(lib.fqkv_decode_plan(0, B, 32, 8, N, 64, 1 << 30, out), "plan")
        if fits64:
            assert out[1] == out[0] >= 2, (B, N, list(out), fits64)
    fqkv.native.check(lib.fqkv_decode_plan(0, 1, 32, 8, 16384, 64, 1 << 30, out), "plan")
    assert out[0] > 1 and out[1] == 0, list(out)
    # a grid of at most 8 units (batch 1) at D = 64 takes the cluster merge up to N = 8192
    fits64 = [c for c in range(2, min(16, sm // 8) + 1) if max_clusters_64[c] >= 8]
    fqkv.native.check(lib.fqkv_decode_plan(0, 1, 32, 8, 8192, 64, 1 << 30, out), "plan")
    if fits64:
        assert out[1] == out[0] >= 2, (list(out), fits64)
    fqkv.native.check(lib.fqkv_decode_plan(0, 2, 32, 8, 8192, 64, 1 << 30, out), "plan")
    assert out[1] == 0, list(out)


@pytest.mark.parametrize("scale", [1e-4, 1e-3, 1e2, "ramp"])
@pytest.mark.parametrize("D", [64, 128])
def test_quantized_kernels_relative_accuracy_at_any_v_scale(fqkv, scale, D):
    """V scaled by 1e-4 .. 1e2 (p * vscale would fall into fp16 subnormals for small V), or by a
    factor rising over the keys from 1e-4 to 1e2 (the V-scale frame moves down inside a unit):
    every quantized kernel -- int8 and int4 with one head per row (the CUDA-core kernel; int4 at
    D = 128 on the tensor cores), int8 GQA on the tensor cores -- within a tolerance relative to
    the output's scale (atol = 2e-3 * scale, or 2e-3 * max|out| for the ramp; rtol = 1e-2) of the
    float64 oracle."""
    R, N = 6, 1500

    def scaled(x, n_axis):
        if scale == "ramp":
            f = torch.logspace(-4, 2, x.shape[n_axis], dtype=torch.float64)
            shape = [1] * x.dim()
            shape[n_axis] = -1
            return (x.double() * f.view(shape)).half(), None
        return (x.float() * scale).half(), scale

    q, K = _randn(R, D, seed=180), _randn(R, N, D, seed=181)
    V, mag = scaled(_randn(R, N, D, seed=182), 1)
    for quant, dq, op in ((fqkv.qpt, oq.dequantize_int8, fqkv.decode_attn_int8_mw),
                          (fqkv.quant_int4_per_token, oq.dequantize_int4, fqkv.decode_attn_int4)):
        Kc, Ks = quant(K.cuda())
        Vc, Vs = quant(V.cuda())
        out = op(q.cuda(), Kc, Vc, Ks, Vs, 8)
        ref = oatt.decode_attention(q.numpy(), dq(Kc.cpu().numpy(), Ks.cpu().numpy()),
                                    dq(Vc.cpu().numpy(), Vs.cpu().numpy()))
        atol = 2e-3 * (mag if mag is not None else np.abs(ref).max())  # ramp: relative to the output's size
        np.testing.assert_allclose(out.float().cpu().numpy().astype(np.float64), ref, atol=atol, rtol=1e-2)
    B, Hq, Hkv = 2, 16, 4
    qg = _randn(B, Hq, D, seed=183)
    Kg = _randn(B, Hkv, N, D, seed=184)
    Vg, mag = scaled(_randn(B, Hkv, N, D, seed=185), 2)
    Kq, Ks = fqkv.qpt(Kg.cuda())
    Vq, Vs = fqkv.qpt(Vg.cuda())
    out = fqkv.decode_attn_gqa_int8(qg.cuda(), Kq, Vq, Ks, Vs)
    ref = oatt.decode_attention_gqa(qg.numpy(), oq.dequantize_int8(Kq.cpu().numpy(), Ks.cpu().numpy()),
                                    oq.dequantize_int8(Vq.cpu().numpy(), Vs.cpu().numpy()))
    atol = 2e-3 * (mag if mag is not None else np.abs(ref).max())
    np.testing.assert_allclose(out.float().cpu().numpy().astype(np.float64), ref, atol=atol, rtol=1e-2)
