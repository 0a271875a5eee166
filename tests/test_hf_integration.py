"""Model integration: the Hugging Face attention hook and the CUDA-graph decode engine.

CPU tests check registration and the prefill hand-off (no GPU needed).  GPU
tests run a small random-weight Llama-architecture model three ways --
``transformers`` with SDPA (the reference's stock path), ``transformers``
with the fqkv hook (the reference's live-model path), and :class:`GraphDecoder`
(static cache, captured decode step) -- and compare them teacher-forced
against SDPA logits on the same token sequence.
"""
from __future__ import annotations

import pytest
import torch


def _tiny_config():
    from transformers import LlamaConfig
    return LlamaConfig(vocab_size=1000, hidden_size=512, intermediate_size=1024, num_hidden_layers=4,
                       num_attention_heads=8, num_key_value_heads=2, head_dim=64, max_position_embeddings=2048,
                       rms_norm_eps=1e-5, rope_theta=500000.0, tie_word_embeddings=True, initializer_range=0.02)


def test_register_adds_hook(fqkv):
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    name = fqkv.hf_integration.register()
    assert name in ALL_ATTENTION_FUNCTIONS


def test_prefill_is_handed_to_sdpa_on_any_device(fqkv):
    from transformers.integrations.sdpa_attention import sdpa_attention_forward

    class M(torch.nn.Module):
        num_key_value_groups = 4
        is_causal = True
    g = torch.Generator().manual_seed(0)
    q = torch.randn(2, 8, 5, 64, generator=g)
    k = torch.randn(2, 2, 5, 64, generator=g)
    v = torch.randn(2, 2, 5, 64, generator=g)
    got, _ = fqkv.hf_integration.kernel_attention_forward(M(), q, k, v, None, scaling=0.125)
    ref, _ = sdpa_attention_forward(M(), q, k, v, None, scaling=0.125)
    torch.testing.assert_close(got, ref)


def test_decode_on_cpu_tensors_has_no_fallback(fqkv):
    q = torch.randn(1, 8, 1, 64)
    k = torch.randn(1, 2, 7, 64)
    with pytest.raises(RuntimeError, match="^cuda"):
        fqkv.hf_integration.kernel_attention_forward(None, q, k, k, None, scaling=0.125)


def _teacher_forced_logits(model, seq):
    with torch.no_grad():
        return model(seq).logits.float()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_graph_decoder_matches_sdpa_teacher_forced(fqkv, dtype):
    from transformers import LlamaForCausalLM
    torch.manual_seed(0)
    with torch.device("cuda"):
        model = LlamaForCausalLM(_tiny_config()).to(dtype).eval()
    model.config._attn_implementation = "sdpa"
    B, P, T = 3, 37, 20
    ids = torch.randint(0, 1000, (B, P), device="cuda")
    dec = fqkv.hf_integration.GraphDecoder(model, batch=B, max_len=P + T, keep_logits=True)
    first = dec.prefill(ids)
    dec.capture()
    steps_logits = [dec.logits.clone()]
    for _ in range(T - 1):
        dec.step()
        steps_logits.append(dec.logits.clone())
    toks = torch.cat([first[:, None], dec.out_tokens[:, P + 1:P + T]], dim=1)          # [B, T]
    seq = torch.cat([ids, toks], dim=1)
    ref = _teacher_forced_logits(model, seq)[:, P - 1:P - 1 + T]                        # logits that chose toks
    ours = torch.stack(steps_logits, dim=1)
    agree = (ref.argmax(-1) == toks).float().mean().item()
    assert agree >= 0.9
    err = (ours - ref).abs().max().item()
    assert err <= 0.02 + 0.03 * ref.abs().max().item()
    dec.prefill(ids)                                   # the same graph again through generate(), which
    assert torch.equal(dec.generate(T - 1), toks[:, 1:])  # also checks the device status word


@pytest.mark.gpu
def test_hf_hook_generate_matches_sdpa(fqkv):
    from transformers import LlamaForCausalLM
    name = fqkv.hf_integration.register()
    torch.manual_seed(1)
    with torch.device("cuda"):
        model = LlamaForCausalLM(_tiny_config()).half().eval()
    ids = torch.randint(0, 1000, (2, 29), device="cuda")
    try:
        model.config._attn_implementation = name
        with torch.no_grad():
            out = model.generate(ids, max_new_tokens=12, do_sample=False, pad_token_id=0)
    finally:
        model.config._attn_implementation = "sdpa"
    gen = out[:, 29:]
    ref = _teacher_forced_logits(model, out)[:, 28:28 + 12].argmax(-1)
    assert (ref == gen).float().mean().item() >= 0.9


@pytest.mark.gpu
def test_graph_decoder_int8_cache_tracks_fp16_cache(fqkv):
    """int8 KV (quantize-on-append in the captured step) against the fp16-cache decoder."""
    from transformers import LlamaForCausalLM
    torch.manual_seed(2)
    with torch.device("cuda"):
        model = LlamaForCausalLM(_tiny_config()).half().eval()
    B, P, T = 2, 41, 16
    ids = torch.randint(0, 1000, (B, P), device="cuda")
    outs = {}
    for kv in ("fp16", "int8"):
        dec = fqkv.hf_integration.GraphDecoder(model, batch=B, max_len=P + T, keep_logits=True, kv_dtype=kv)
        dec.prefill(ids)
        dec.capture()
        logits = [dec.logits.clone()]
        for _ in range(T - 1):
            dec.step()
            logits.append(dec.logits.clone())
        outs[kv] = (torch.stack(logits, 1), dec.out_tokens[:, P:P + T].clone())
    (l16, t16), (l8, t8) = outs["fp16"], outs["int8"]
    # int8 KV perturbs attention by ~1 % (per-token quantization); the step must
    # stay close to the fp16-cache step on the same model
    assert (t16 == t8).float().mean().item() >= 0.75
    first_div = int((t16 != t8).any(0).float().argmax()) if (t16 != t8).any() else T
    err = (l8[:, :max(first_div, 1)] - l16[:, :max(first_div, 1)]).abs().max().item()
    assert err <= 0.05 + 0.05 * l16.abs().max().item()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("kv", ["fp16", "int8"])
def test_rope_qkv_append_bit_exact(fqkv, dtype, kv):
    """The fused prologue equals transformers' RoPE + .to(float16) + cache append / qpt, bit for bit."""
    from transformers import LlamaForCausalLM
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    torch.manual_seed(4)
    with torch.device("cuda"):
        model = LlamaForCausalLM(_tiny_config()).to(dtype).eval()
    rot = model.model.rotary_emb
    B, Hq, Hkv, D, cap, pos = 3, 8, 2, 64, 50, 37
    qkv = (torch.randn(B, (Hq + 2 * Hkv) * D, device="cuda") * 3).to(dtype)
    cos_t, sin_t = rot(torch.empty(1, 1, 1, dtype=dtype, device="cuda"), torch.arange(cap, device="cuda")[None])
    cos_t, sin_t = cos_t[0].contiguous(), sin_t[0].contiguous()
    q_out = torch.empty(B, Hq, D, dtype=torch.float16, device="cuda")
    cdt = torch.float16 if kv == "fp16" else torch.int8
    K = torch.zeros(B, Hkv, cap, D, dtype=cdt, device="cuda")
    V = torch.zeros_like(K)
    Ks = torch.zeros(B, Hkv, cap, dtype=torch.float16, device="cuda") if kv == "int8" else None
    Vs = torch.zeros_like(Ks) if kv == "int8" else None
    posd = torch.tensor([pos], dtype=torch.int32, device="cuda")
    fqkv.rope_qkv_append(qkv, cos_t, sin_t, posd, q_out, K, V, Ks, Vs)
    # reference: the HF ops the decoder used before
    q = qkv[:, :Hq * D].view(B, 1, Hq, D).transpose(1, 2)
    k = qkv[:, Hq * D:(Hq + Hkv) * D].view(B, 1, Hkv, D).transpose(1, 2)
    v = qkv[:, (Hq + Hkv) * D:].view(B, 1, Hkv, D).transpose(1, 2)
    cos, sin = rot(qkv[:, None], torch.full((B, 1), pos, device="cuda"))
    qr, kr = apply_rotary_pos_emb(q, k, cos, sin)
    assert torch.equal(q_out, qr[:, :, 0].to(torch.float16))
    k16, v16 = kr[:, :, 0].to(torch.float16), v[:, :, 0].to(torch.float16)
    if kv == "fp16":
        assert torch.equal(K[:, :, pos], k16) and torch.equal(V[:, :, pos], v16)
    else:
        kc, ksc = fqkv.qpt(k16.contiguous())
        vc, vsc = fqkv.qpt(v16.contiguous())
        assert torch.equal(K[:, :, pos], kc) and torch.equal(V[:, :, pos], vc)
        assert torch.equal(Ks[:, :, pos], ksc) and torch.equal(Vs[:, :, pos], vsc)
    assert not K[:, :, :pos].any() and not K[:, :, pos + 1:].any()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("D,bias", [(64, False), (128, True)])
def test_gemv_rope_append_equals_gemv_then_rope_append(fqkv, dtype, D, bias):
    """The batch-1 q/k/v GEMV with RoPE, q cast and fp16 cache append in its epilogue: the same q and
    cache rows as the GEMV followed by rope_qkv_append (itself bit-exact with transformers' RoPE), with
    a device or host position; a position past the cache writes q only."""
    torch.manual_seed(D + bias)
    Hq, Hkv, Hid, cap, rows = 8, 2, 512, 40, 64
    x = torch.randn(1, Hid, device="cuda").to(dtype)
    W = (torch.randn((Hq + 2 * Hkv) * D, Hid, device="cuda") * 0.05).to(dtype)
    b = torch.randn(W.shape[0], device="cuda").to(dtype) if bias else None
    ang = torch.arange(rows, device="cuda")[:, None] * torch.linspace(0.01, 1.0, D // 2, device="cuda")[None]
    cos_t = torch.cat([ang.cos(), ang.cos()], 1).to(dtype).contiguous()
    sin_t = torch.cat([ang.sin(), ang.sin()], 1).to(dtype).contiguous()
    for pos in (torch.tensor([7], dtype=torch.int32, device="cuda"), 39, 45):
        outs = []
        for fused in (True, False):
            q = torch.full((1, Hq, D), float("nan"), dtype=torch.float16, device="cuda")
            K = torch.zeros(1, Hkv, cap, D, dtype=torch.float16, device="cuda")
            V = torch.zeros_like(K)
            if fused:
                fqkv.gemv_rope_append(x, W, b, cos_t, sin_t, pos, q, K, V)
            else:
                fqkv.rope_qkv_append(fqkv.gemv(x, W, b), cos_t, sin_t, pos, q, K, V)
            outs.append((q, K, V))
        (qf, Kf, Vf), (qr, Kr, Vr) = outs
        assert torch.equal(qf, qr) and torch.equal(Kf, Kr) and torch.equal(Vf, Vr), pos
        if pos == 45:   # past the cache: q written, the cache untouched
            assert torch.isfinite(qf).all() and not Kf.any() and not Vf.any()


@pytest.mark.gpu
@pytest.mark.parametrize("kv", ["fp16", "int8"])
def test_graph_decoder_fused_prologue_equals_hf_ops(fqkv, kv):
    """GraphDecoder with the fused RoPE/append prologue gives the same logits, bit for bit,
    as with transformers' RoPE and separate cache writes."""
    from transformers import LlamaForCausalLM
    torch.manual_seed(6)
    with torch.device("cuda"):
        model = LlamaForCausalLM(_tiny_config()).to(torch.bfloat16).eval()
    B, P, T = 2, 29, 10
    ids = torch.randint(0, 1000, (B, P), device="cuda")
    res = {}
    for fused in (False, True):
        dec = fqkv.hf_integration.GraphDecoder(model, batch=B, max_len=P + T, keep_logits=True, kv_dtype=kv,
                                               fused_rope=fused, fused_model_ops=False)
        assert dec.rope_fused == fused
        dec.prefill(ids)
        dec.capture()
        lg = [dec.logits.clone()]
        for _ in range(T - 1):
            dec.step()
            lg.append(dec.logits.clone())
        res[fused] = torch.stack(lg, 1)
    assert torch.equal(res[False], res[True])


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("B", [2, 8])
def test_graph_decoder_fused_model_ops_track_hf_modules(fqkv, dtype, B):
    """The fused residual/RMSNorm + SwiGLU step against transformers' modules on
    the same decoder: same tokens, logits within rounding (the RMSNorm sum of
    squares and the concatenated gate/up GEMM reduce in a different order; a
    bf16 model at batch > 4 also takes the attention output in bf16)."""
    from transformers import LlamaForCausalLM
    torch.manual_seed(8)
    with torch.device("cuda"):
        model = LlamaForCausalLM(_tiny_config()).to(dtype).eval()
    P, T = 31, 12
    ids = torch.randint(0, 1000, (B, P), device="cuda")
    res = {}
    for fused in (False, True):
        dec = fqkv.hf_integration.GraphDecoder(model, batch=B, max_len=P + T, keep_logits=True,
                                               fused_model_ops=fused)
        assert dec.model_fused == fused
        if fused and dtype == torch.bfloat16 and B > 4:
            assert dec.attn_out.dtype == torch.bfloat16
        dec.prefill(ids)
        dec.capture()
        lg = [dec.logits.clone()]
        for _ in range(T - 1):
            dec.step()
            lg.append(dec.logits.clone())
        res[fused] = (torch.stack(lg, 1), dec.out_tokens[:, P:P + T].clone())
    (l0, t0), (l1, t1) = res[False], res[True]
    assert (t0 == t1).float().mean().item() >= 0.9
    n_ok = int((t0 != t1).any(0).float().argmax()) if (t0 != t1).any() else T
    err = (l1[:, :max(n_ok, 1)] - l0[:, :max(n_ok, 1)]).abs().max().item()
    assert err <= 0.02 + 0.01 * l0.abs().max().item()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("H", [2048, 520])
def test_add_rmsnorm_and_silu_mul_kernels(fqkv, dtype, H):
    """Residual add bit-exact; RMSNorm within one unit in the last place of the
    model dtype of transformers' LlamaRMSNorm (only the fp32 sum order differs);
    SwiGLU bit-exact with torch's silu(g) * u.  H=520 takes the scalar path."""
    from transformers.models.llama.modeling_llama import LlamaRMSNorm
    torch.manual_seed(9)
    rows = 7
    h = (torch.randn(rows, H, device="cuda") * 2).to(dtype)
    d = torch.randn(rows, H, device="cuda").to(dtype)
    norm = LlamaRMSNorm(H, eps=1e-5).cuda().to(dtype)
    with torch.no_grad():
        norm.weight.copy_((1 + 0.1 * torch.randn(H, device="cuda")).to(dtype))
        h_ref = h + d
        y_ref = norm(h_ref)
    y = torch.empty_like(h)
    fqkv.add_rmsnorm(h, d, norm.weight.detach(), y, 1e-5)
    assert torch.equal(h, h_ref)
    ulp = torch.finfo(dtype).eps * y_ref.float().abs().clamp_min(torch.finfo(dtype).tiny)
    assert ((y.float() - y_ref.float()).abs() <= ulp * 1.01).all()
    assert (y == y_ref).float().mean().item() >= 0.97
    y2 = torch.empty_like(h)
    fqkv.add_rmsnorm(h, None, norm.weight.detach(), y2, 1e-5)   # plain norm of the updated stream
    assert torch.equal(y2, y)
    for I in (300, 2048):   # scalar path, 16-byte path
        gu = (torch.randn(rows, 2 * I, device="cuda") * 3).to(dtype)
        out = torch.empty(rows, I, device="cuda", dtype=dtype)
        fqkv.silu_mul(gu, out)
        assert torch.equal(out, torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]), I


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("B,N,K", [(1, 300, 512), (2, 1000, 2048), (3, 77, 8192), (4, 2048, 2048), (1, 3, 256)])
def test_gemv_matches_fp32_projection(fqkv, dtype, B, N, K):
    """Small-batch GEMV: within one output rounding of the fp32 product (with bias)."""
    torch.manual_seed(B * 1000 + N)
    x = torch.randn(B, K, device="cuda").to(dtype)
    W = (torch.randn(N, K, device="cuda") * 0.05).to(dtype)
    b = torch.randn(N, device="cuda").to(dtype)
    ref = x.float() @ W.float().t() + b.float()
    got = fqkv.gemv(x, W, b).float()
    tol = torch.finfo(dtype).eps * ref.abs() + 1e-4 * ref.abs().max()
    assert ((got - ref).abs() <= tol).all()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("B,I,K,bias", [(1, 8192, 2048, False), (4, 300, 2048, True), (2, 77, 512, True),
                                         (3, 1000, 4096, False)])
def test_gemv_swiglu_equals_gemv_then_silu_mul(fqkv, dtype, B, I, K, bias):
    """The fused gate/up GEMV + SwiGLU: bit-identical to the GEMV of [gate; up] followed by the SwiGLU
    kernel (the same per-row dot products and roundings) wherever that GEMV runs one warp per row
    (K <= 2048, or any K at B > 1); at B = 1 with K > 2048 the plain GEMV sums K-slices in another
    order, so there it is checked within one output rounding.  And against the fp32 reference of
    silu(x Wg^T + bg) * (x Wu^T + bu)."""
    torch.manual_seed(B * 7 + I)
    x = torch.randn(B, K, device="cuda").to(dtype)
    W = (torch.randn(2 * I, K, device="cuda") * 0.05).to(dtype)
    b = torch.randn(2 * I, device="cuda").to(dtype) if bias else None
    got = fqkv.gemv_swiglu(x, W, b)
    assert got.shape == (B, I) and got.dtype == dtype
    two = torch.empty(B, I, device="cuda", dtype=dtype)
    fqkv.silu_mul(fqkv.gemv(x, W, b), two)
    if K <= 2048 or B > 1:
        assert torch.equal(got, two)
    else:
        assert ((got.float() - two.float()).abs() <= 2 * torch.finfo(dtype).eps * two.float().abs() + 1e-6).all()
    g = x.float() @ W[:I].float().t() + (b[:I].float() if bias else 0)
    u = x.float() @ W[I:].float().t() + (b[I:].float() if bias else 0)
    ref = torch.nn.functional.silu(g) * u
    tol = 4 * torch.finfo(dtype).eps * ref.abs() + 1e-3 * ref.abs().max()
    assert ((got.float() - ref).abs() <= tol).all()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("rows,V", [(1, 128256), (4, 32000), (64, 128256), (3, 100), (2, 1), (2, 16), (300, 1000)])
def test_argmax_rows_matches_torch(fqkv, dtype, rows, V):
    """Multi-CTA argmax: the same index as torch.argmax, ties to the first index, reusable scratch."""
    from importlib import import_module
    native = import_module(fqkv.__name__ + "._native")

    torch.manual_seed(rows * 7 + V)
    scratch = torch.zeros(int(native.lib().fqkv_argmax_scratch_bytes(rows)), dtype=torch.uint8, device="cuda")
    for trial in range(3):
        x = (torch.randn(rows, V, device="cuda") * 4).to(dtype)
        if trial == 1 and V > 8:
            # ties: the maximum repeated in several slices of the row
            m = x.float().max() + 1
            x[:, V // 3] = m.to(dtype)
            x[:, V - 1] = m.to(dtype)
            x[:, V // 7 + 1] = m.to(dtype)
        if trial == 2:
            x[0, V // 2] = float("nan")
            if V > 4:
                x[0, V - 1] = float("nan")
        got = fqkv.ops.argmax_rows(x, scratch)
        assert torch.equal(got.cpu(), x.argmax(-1).cpu()), trial


@pytest.mark.gpu
@pytest.mark.parametrize("B,N,K", [(1, 2048, 2048), (3, 300, 512), (4, 77, 4096)])
def test_gemv_fp16_activations_bf16_weights_equal_cast_first(fqkv, B, N, K):
    """fp16 x with bf16 W: bit-identical to casting x to bf16 before the GEMV."""
    torch.manual_seed(N + K)
    x = (torch.randn(B, K, device="cuda") * 3).half()
    W = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    b = torch.randn(N, device="cuda").bfloat16()
    got = fqkv.gemv(x, W, b)
    assert got.dtype == torch.bfloat16
    assert torch.equal(got, fqkv.gemv(x.to(torch.bfloat16), W, b))
