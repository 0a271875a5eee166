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
