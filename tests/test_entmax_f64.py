"""CPU checks of the float64 α-entmax reference (tests/entmax_f64.py) that
the exact-threshold and Jacobian GPU tests compare against."""
import pytest
import torch

from entmax_f64 import entmax_attention


@pytest.mark.parametrize("alpha", [1.5, 2.0, 1.25])
def test_rows_sum_to_one_and_match_sparsemax(alpha):
    g = torch.Generator().manual_seed(0)
    Q, K, V = (torch.randn(1, 16, 8, generator=g, dtype=torch.float64) for _ in range(3))
    idx = torch.arange(16).expand(1, 16)
    O, tau = entmax_attention(Q, K, V, idx, idx, alpha, 0.5, causal=True)
    s = torch.clamp(0.5 * Q @ K.transpose(1, 2), -10, 10)
    vis = idx[:, None, :] <= idx[:, :, None]
    p = torch.clamp((alpha - 1) * s - tau[..., None], min=0) ** (1 / (alpha - 1)) * vis
    assert torch.allclose(p.sum(-1), torch.ones(1, 16, dtype=torch.float64), atol=1e-9)
    if alpha == 2.0:   # sparsemax closed form from the sorted scores
        for r in range(16):
            z = s[0, r, : r + 1].sort(descending=True).values
            css = z.cumsum(0)
            k = torch.arange(1, r + 2, dtype=torch.float64)
            supp = (1 + k * z > css).nonzero().max() + 1
            t = (css[supp - 1] - 1) / supp
            assert abs(float(t) - float(tau[0, r])) < 1e-9


@pytest.mark.parametrize("alpha", [1.5, 2.0])
def test_gradient_matches_finite_differences(alpha):
    g = torch.Generator().manual_seed(1)
    Q, K, V, dO = (torch.randn(1, 12, 6, generator=g, dtype=torch.float64) for _ in range(4))
    idx = torch.arange(12).expand(1, 12)
    Q.requires_grad_()
    O, _ = entmax_attention(Q, K, V, idx, idx, alpha, 0.7)
    (O * dO).sum().backward()
    eps = 1e-6
    for (r, c) in [(3, 1), (7, 4), (11, 0), (5, 5)]:
        Qp, Qm = Q.detach().clone(), Q.detach().clone()
        Qp[0, r, c] += eps
        Qm[0, r, c] -= eps
        fp = (entmax_attention(Qp, K, V, idx, idx, alpha, 0.7)[0] * dO).sum()
        fm = (entmax_attention(Qm, K, V, idx, idx, alpha, 0.7)[0] * dO).sum()
        fd = float((fp - fm) / (2 * eps))
        assert abs(fd - float(Q.grad[0, r, c])) < 1e-6 * max(1.0, abs(fd))
