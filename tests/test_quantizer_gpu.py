"""GPU quantizers: bit-exact against the reference's outputs and the oracle.

* The golden vectors (produced by the reference's own ``qpt`` /
  ``quant_int4_per_token``) must be reproduced exactly, edge tokens included.
* Large random inputs: bit-exact against the numpy restatement.
* The reference quantizer expression evaluated by torch on CUDA tensors (the
  way the reference's tests run ``qpt``) must agree bit-for-bit too.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import quant as oq

pytestmark = pytest.mark.gpu


def _fp16_equal(a: np.ndarray, b: np.ndarray) -> bool:
    a = np.asarray(a, np.float16)
    b = np.asarray(b, np.float16)
    if not np.array_equal(np.isnan(a), np.isnan(b)):
        return False
    m = ~np.isnan(a)
    return np.array_equal(a.view(np.uint16)[m], b.view(np.uint16)[m])


@pytest.fixture(scope="module")
def qg(golden_dir):
    return dict(np.load(golden_dir / "quant_golden.npz"))


@pytest.mark.parametrize("tag", ["rand", "edge"])
@pytest.mark.parametrize("D", [64, 128])
def test_golden_int8(fqkv, qg, tag, D):
    X = torch.from_numpy(qg[f"X_{tag}_D{D}"]).cuda()
    c, s = fqkv.qpt(X)
    assert np.array_equal(c.cpu().numpy(), qg[f"codes8_{tag}_D{D}"])
    assert _fp16_equal(s.cpu().numpy(), qg[f"scales8_{tag}_D{D}"])


@pytest.mark.parametrize("tag", ["rand", "edge"])
@pytest.mark.parametrize("D", [64, 128])
def test_golden_int4(fqkv, qg, tag, D):
    X = torch.from_numpy(qg[f"X_{tag}_D{D}"]).cuda()
    p, s = fqkv.quant_int4_per_token(X)
    assert np.array_equal(p.cpu().numpy(), qg[f"packed4_{tag}_D{D}"])
    assert _fp16_equal(s.cpu().numpy(), qg[f"scales4_{tag}_D{D}"])


@pytest.mark.parametrize("D", [64, 128, 256, 96, 30, 7])
def test_random_bit_exact_vs_oracle(fqkv, D):
    g = torch.Generator().manual_seed(D)
    X = (torch.randn(37, 129, D, generator=g) * torch.rand(37, 129, 1, generator=g) * 4).to(torch.float16)
    c8, s8 = fqkv.qpt(X.cuda())
    rc8, rs8 = oq.quantize_int8_per_token(X.numpy())
    assert np.array_equal(c8.cpu().numpy(), rc8)
    assert _fp16_equal(s8.cpu().numpy(), rs8)
    if D % 2 == 0:
        p4, s4 = fqkv.quant_int4_per_token(X.cuda())
        rp4, rs4 = oq.quantize_int4_per_token(X.numpy())
        assert np.array_equal(p4.cpu().numpy(), rp4)
        assert _fp16_equal(s4.cpu().numpy(), rs4)


def _reference_expression_cuda(X: torch.Tensor, qmax: float):
    """The reference quantizer's torch arithmetic, evaluated on CUDA tensors."""
    a = X.abs().amax(-1, keepdim=True)
    s = (a / qmax).clamp(min=1e-8)
    codes = torch.clamp(torch.round(X / s), -qmax, qmax).to(torch.int8)
    return codes, s.squeeze(-1)


@pytest.mark.parametrize("D", [64, 128])
def test_matches_torch_cuda_evaluation(fqkv, D):
    gen = torch.Generator(device="cuda").manual_seed(123)
    X = torch.randn(64, 1000, D, device="cuda", generator=gen, dtype=torch.float16)
    X[0, :5] = 0
    X[1, 3, 7] = 0.5 * 127 / 127  # exact-half ties after division
    c8, s8 = fqkv.qpt(X)
    rc8, rs8 = _reference_expression_cuda(X, 127.0)
    assert torch.equal(c8, rc8)
    assert torch.equal(s8.view(torch.int16), rs8.view(torch.int16))
    p4, s4 = fqkv.quant_int4_per_token(X)
    rc4, rs4 = _reference_expression_cuda(X, 7.0)
    assert torch.equal(s4.view(torch.int16), rs4.view(torch.int16))
    assert np.array_equal(p4.cpu().numpy(), oq.pack_int4(rc4.cpu().numpy()))


def test_empty_and_large_row_counts(fqkv):
    X = torch.empty(0, 128, dtype=torch.float16, device="cuda")
    c, s = fqkv.qpt(X)
    assert c.shape == (0, 128) and s.shape == (0,)
    X = torch.randn(8, 32, 4096, 128, dtype=torch.float16, device="cuda")
    c, s = fqkv.qpt(X)
    i = torch.randint(0, 8 * 32 * 4096, (512,))
    Xs = X.view(-1, 128)[i].cpu().numpy()
    rc, rs = oq.quantize_int8_per_token(Xs)
    assert np.array_equal(c.view(-1, 128)[i].cpu().numpy(), rc)
    assert _fp16_equal(s.view(-1)[i].cpu().numpy(), rs)


def _every_fp16_pair_tokens(dev):
    """Tokens of D=128 covering every pair (a, x) of fp16 values with a > 0 finite and |x| <= a:
    element 0 of a token is a (its largest magnitude, so the token's scale is fp16(a / Q)), the
    other 127 are consecutive fp16 bit patterns 0 .. a of x (the last token of each a padded with a).
    About 4M tokens (1 GiB); the same tokens negated cover x < 0."""
    per = 127
    a_bits = torch.arange(1, 0x7C00, device=dev, dtype=torch.int64)          # positive finite fp16
    ntok = (a_bits + per) // per                                             # ceil((a_bits + 1) / 127)
    tok_a = torch.repeat_interleave(a_bits, ntok)
    first = torch.cumsum(ntok, 0) - ntok
    tok_j = torch.arange(tok_a.numel(), device=dev) - torch.repeat_interleave(first, ntok)
    xp = torch.minimum(tok_j[:, None] * per + torch.arange(per, device=dev)[None, :], tok_a[:, None])
    return torch.cat([tok_a[:, None], xp], 1).to(torch.int16).view(torch.float16).contiguous()


def _reference_expression(X: torch.Tensor, Q: int):
    """The reference quantizer (notebook lines 236-238 / 292-299) as torch evaluates it on CUDA tensors;
    NaN codes (0 / 0 in a token whose scale underflowed) -> 0 as .to(int8) gives on the CPU."""
    a = X.abs().amax(-1, keepdim=True)
    s = (a / Q).clamp(min=1e-8)
    r = torch.clamp(torch.round(X / s), -Q, Q)
    return torch.where(torch.isnan(r), torch.zeros_like(r), r).to(torch.int8), s.squeeze(-1)


def test_every_fp16_pair_bit_exact(fqkv):
    """Codes and scales bit-exact with the reference expression for every (amax, x) fp16 pair, both
    signs, int8 and int4: the kernel's division (FMA-corrected reciprocal for normal scales, IEEE
    division otherwise) must round exactly as the IEEE quotient everywhere."""
    dev = "cuda"
    Xp = _every_fp16_pair_tokens(dev)
    for X in (Xp, -Xp):
        c8, s8 = fqkv.qpt(X)
        r8, rs = _reference_expression(X, 127)
        assert torch.equal(s8.view(torch.int16), rs.view(torch.int16))
        bad = (c8 != r8).sum().item()
        assert bad == 0, f"{bad} int8 codes differ"
        p4, s4 = fqkv.quant_int4_per_token(X)
        r4, rs4 = _reference_expression(X, 7)
        assert torch.equal(s4.view(torch.int16), rs4.view(torch.int16))
        lo = (p4 & 0xF).to(torch.int8)
        hi = (p4 >> 4).to(torch.int8)
        unpacked = torch.stack([torch.where(lo >= 8, lo - 16, lo), torch.where(hi >= 8, hi - 16, hi)], -1).flatten(-2)
        bad = (unpacked != r4).sum().item()
        assert bad == 0, f"{bad} int4 codes differ"
        del c8, r8, p4, r4, lo, hi, unpacked
    # and a slice against the numpy restatement (IEEE fp32 division on the CPU)
    idx = torch.randint(0, Xp.shape[0], (20000,), device=dev, generator=torch.Generator(device=dev).manual_seed(9))
    Xs = Xp[idx]
    c8, s8 = fqkv.qpt(Xs)
    rc, rsc = oq.quantize_int8_per_token(Xs.cpu().numpy())
    assert np.array_equal(c8.cpu().numpy(), rc) and _fp16_equal(s8.cpu().numpy(), rsc)
