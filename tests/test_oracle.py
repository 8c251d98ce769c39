"""Known-answer tests of the CPU oracle (oracle/asa_oracle.c) against facts
derived from the reference's formulas (source/adasplashattention.cu)."""
import numpy as np
import pytest
import torch

from helpers import make_inputs, oracle_run
from oracle import oracle as orc


def test_first_query_attends_only_key0():
    # causal arange: query 0 sees key 0 alone, so O[0] = p v0 / (p + 1e-8) = v0
    Q, K, V, dO, Qi, Ki = make_inputs(1, 2, 128, 128, 64, seed=3)
    r = oracle_run(Q, K, V, dO, Qi, Ki, 64, 64, 8, 1.5, 0.125, grads=False)
    np.testing.assert_allclose(r["O"][:, 0], V[0, :, 0].numpy(), atol=1e-6)


def test_topk_tie_break_keeps_earliest_keys():
    # identical keys => identical scores; strict '>' keeps the first k keys (:35-49)
    d, N = 32, 96
    Q = torch.randn(1, 1, N, d)
    K = torch.randn(1, 1, 1, d).expand(1, 1, N, d).contiguous()
    cfg = orc.Config(1, N, N, d, 32, 32, 8, 1.5, 0.125, causal=False)
    Qi = np.full((1, N), 2 ** 31 - 1, np.int32)
    Ki = np.arange(N, dtype=np.int32)[None]
    tau, M, topv, topi = orc.tau_mask(cfg, Q.numpy().reshape(1, N, d), K.numpy().reshape(1, N, d),
                                      Qi, Ki, want_topk=True)
    assert (topi == np.arange(8)[None, None]).all()
    assert M[0, :, 0].all() and not M[0, :, 1:].any()


def test_sentinel_rows_keep_minus_1e6():
    # rows with fewer than k visible keys keep (-1e6, -1) sentinels (:166-172)
    Q, K, V, dO, Qi, Ki = make_inputs(1, 1, 64, 64, 32, seed=1)
    cfg = orc.Config(1, 64, 64, 32, 32, 32, 8, 1.5, 32 ** -0.5)
    tau, M, topv, topi = orc.tau_mask(cfg, Q.numpy()[0], K.numpy()[0], Qi.numpy(), Ki.numpy(),
                                      want_topk=True)
    for q in range(7):
        assert (topi[0, q, q + 1:] == -1).all() and (topv[0, q, q + 1:] == -1e6).all()
        assert sorted(topi[0, q, :q + 1]) == list(range(q + 1))
    assert (topi[0, 7:] >= 0).all()
    # the sentinels widen the bracket to ~(α-1)·(-1e6); five steps leave τ far
    # below every real score, so those rows are close to uniform
    assert (tau[0, :7] < -20).all() and (tau[0, 7:] > -20).all()


def _sparsemax_tau(z):
    z = np.sort(z)[::-1].astype(np.float64)
    cs = np.cumsum(z)
    r = np.arange(1, len(z) + 1)
    support = z - (cs - 1) / r > 0
    k = r[support][-1]
    return (cs[k - 1] - 1) / k


def test_alpha2_matches_closed_form_sparsemax():
    # α=2: f is piecewise linear, c2 = 0 so Halley is Newton; where the five
    # steps reached |f| < 1e-4 the result is the sparsemax threshold.
    rng = np.random.default_rng(0)
    checked = 0
    for _ in range(300):
        s = np.sort(rng.normal(0, 1.5, 8).astype(np.float32))[::-1].copy()
        tau = orc.entmax_tau(s, 2.0)
        f = np.maximum(s.astype(np.float64) - tau, 0).sum() - 1
        if abs(f) < 1e-4:
            assert abs(tau - _sparsemax_tau(s)) < 2e-4
            checked += 1
    assert checked > 200


def test_alpha_is_clamped():
    s = np.array([3, 2, 1, 0.5, 0, -1, -2, -3], np.float32)
    assert orc.entmax_tau(s, 0.5) == orc.entmax_tau(s, 1.05)
    assert orc.entmax_tau(s, 7.0) == orc.entmax_tau(s, 3.0)


def test_csr_matches_mask():
    rng = np.random.default_rng(1)
    cfg = orc.Config(3, 200, 300, 16, 32, 64)
    M = (rng.random((3, cfg.nQB, cfg.nKB)) < 0.4).astype(np.uint8)
    ptr, idx = orc.csr(cfg, M)
    for b in range(3):
        assert ptr[b, 0] == 0
        for i in range(cfg.nQB):
            assert list(idx[b, ptr[b, i]:ptr[b, i + 1]]) == list(np.nonzero(M[b, i])[0])
        assert (idx[b, ptr[b, -1]:] == 0).all()


@pytest.mark.parametrize("alpha", [1.5, 2.0, 1.25])
def test_backward_is_fixed_tau_gradient(alpha):
    # The reference backward (:439-523) is the exact gradient of Σ O·dO with τ
    # and the mask held fixed.  Check against torch float64 autograd of the
    # same objective (scores kept inside ±10 so the ungated clamp is moot).
    B, H, N, d, BM, BN = 1, 2, 96, 16, 32, 32
    Q, K, V, dO, Qi, Ki = make_inputs(B, H, N, N, d, seed=5, sigma=0.7)
    sc = 0.3
    r = oracle_run(Q, K, V, dO, Qi, Ki, BM, BN, 8, alpha, sc, ref_tile_load=False)
    tau = torch.from_numpy(r["tau"]).double()
    act = torch.from_numpy(r["M"]).bool()
    q, k, v = (x.double().reshape(B * H, N, d).requires_grad_() for x in (Q, K, V))
    s = torch.clamp(q @ k.transpose(1, 2) * sc, -10, 10)
    vis = torch.tril(torch.ones(N, N, dtype=torch.bool))
    tile = act.repeat_interleave(BM, 1).repeat_interleave(BN, 2)[:, :N, :N]
    u = (alpha - 1) * s - tau[:, :, None]
    p = torch.where(vis & tile & (u > 0), torch.clamp(u, min=1e-8) ** (1 / (alpha - 1)), 0.0)
    O = (p @ v) / (p.sum(-1, keepdim=True) + 1e-8)
    (O * dO.double().reshape(B * H, N, d)).sum().backward()
    for name, g in (("dQ", q.grad), ("dK", k.grad), ("dV", v.grad)):
        ref = g.numpy()
        err = np.abs(r[name] - ref).max() / max(1.0, np.abs(ref).max())
        assert err < 1e-4, (name, err)


def test_forward_matches_dense_restatement():
    Q, K, V, dO, Qi, Ki = make_inputs(1, 2, 160, 160, 32, seed=7)
    r = oracle_run(Q, K, V, dO, Qi, Ki, 32, 64, 8, 1.5, 0.2, grads=False, ref_tile_load=False)
    BH, N, d = 2, 160, 32
    q, k, v = (x.double().reshape(BH, N, d) for x in (Q, K, V))
    s = torch.clamp(q @ k.transpose(1, 2) * 0.2, -10, 10)
    vis = torch.tril(torch.ones(N, N, dtype=torch.bool))
    act = torch.from_numpy(r["M"]).bool().repeat_interleave(32, 1).repeat_interleave(64, 2)[:, :N, :N]
    u = 0.5 * s - torch.from_numpy(r["tau"]).double()[:, :, None]
    p = torch.where(vis & act & (u > 0), u.clamp(min=1e-8) ** 2, 0.0)
    O = (p @ v) / (p.sum(-1, keepdim=True) + 1e-8)
    np.testing.assert_allclose(r["O"], O.numpy(), atol=2e-5)
