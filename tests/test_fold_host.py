"""LayerNorm folded into a linear layer (forgeml_b200.linear.ln_fold_vectors),
checked on the CPU in float64: the decode GEMM computes
    rstd * (x W'^T - mean * wsum) + wbias,   W' = W diag(gamma),
which must equal LayerNorm(x) W^T (F.layer_norm, biased variance)."""

import torch

from forgeml_b200.linear import ln_fold_vectors


def _ln_linear(x, w, g, b, eps):
    return torch.nn.functional.layer_norm(x, (x.shape[1],), g, b, eps) @ w.t()


def _folded(x, w, g, b, eps):
    wp, wsum, wbias = ln_fold_vectors(w, g, b)
    mean = x.mean(dim=1, keepdim=True)
    var = x.var(dim=1, unbiased=False, keepdim=True)
    rstd = 1.0 / torch.sqrt(var + eps)
    y = rstd * (x @ wp.t() - mean * wsum.to(x.dtype)[None, :])
    if wbias is not None:
        y = y + wbias.to(x.dtype)[None, :]
    return y, wp, wbias


def test_fold_equals_layernorm_then_linear():
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(7, 96, generator=gen, dtype=torch.float64) * 2 + 0.5
    w = torch.randn(40, 96, generator=gen, dtype=torch.float64) * 0.05
    g = 1 + 0.2 * torch.randn(96, generator=gen, dtype=torch.float64)
    b = 0.1 * torch.randn(96, generator=gen, dtype=torch.float64)
    got, wp, wbias = _folded(x, w, g, b, 1e-5)
    # the sums are formed in fp32 by ln_fold_vectors
    torch.testing.assert_close(got, _ln_linear(x, w, g, b, 1e-5), rtol=1e-5, atol=1e-5)
    assert wp is not w and wbias is not None


def test_identity_layernorm_reuses_the_weight():
    gen = torch.Generator().manual_seed(1)
    w = (torch.randn(16, 64, generator=gen) * 0.02).to(torch.bfloat16)
    wp, wsum, wbias = ln_fold_vectors(w, torch.ones(64, dtype=torch.bfloat16), torch.zeros(64, dtype=torch.bfloat16))
    assert wp is w and wbias is None
    assert wsum.dtype == torch.float32
    torch.testing.assert_close(wsum, w.float().sum(dim=1))


def test_gamma_is_folded_into_the_weight_dtype():
    gen = torch.Generator().manual_seed(2)
    w = (torch.randn(8, 32, generator=gen) * 0.02).to(torch.bfloat16)
    g = (1 + 0.1 * torch.randn(32, generator=gen)).to(torch.bfloat16)
    wp, wsum, _ = ln_fold_vectors(w, g, torch.zeros(32, dtype=torch.bfloat16))
    assert wp.dtype == torch.bfloat16 and wp.is_contiguous()
    torch.testing.assert_close(wp, (w.float() * g.float()).to(torch.bfloat16))
    torch.testing.assert_close(wsum, wp.float().sum(dim=1))
