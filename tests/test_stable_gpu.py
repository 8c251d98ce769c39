"""The top-k-only ("stable") operator of the reference notebook
(AdaSplashNotebook.ipynb file lines 303-450): forward against the C oracle
(oracle/asa_oracle.c asa_oracle_stable_forward), gradient against float64
torch autograd of the same algorithm (tests/stable_f64.py); the notebook's
own backward returns zeros."""
import numpy as np
import pytest
import torch

from helpers import make_inputs, assert_close, OUT_ATOL
from oracle import oracle as orc
from stable_f64 import stable_attention_f64

pytestmark = pytest.mark.gpu

# name: dtype, d, alpha, sm_scale, k, causal, sigma
CASES = {
    "fp32_a15": (torch.float32, 64, 1.5, 0.125, 8, True, 1.0),
    "fp32_a2_k16": (torch.float32, 64, 2.0, 0.125, 16, True, 1.0),
    "fp32_a13_noncausal": (torch.float32, 48, 1.3, 0.2, 8, False, 1.0),
    "bf16_tc_d128": (torch.bfloat16, 128, 1.5, 128 ** -0.5, 8, True, 1.0),
    "bf16_tc_d64_a2": (torch.bfloat16, 64, 2.0, 0.125, 8, True, 1.0),
}


def engine(Q, K, V, dO, Qi, Ki, alpha, sc, k, causal, cuda):
    from splash_attention import ops
    st = ops.Settings(alpha=alpha, sm_scale=sc, k_keep=k, causal=causal, out_dtype=torch.float32,
                      ref_tile_load=False)
    dev = [x.to(cuda) for x in (Q, K, V, dO, Qi, Ki)]
    O, s = ops.stable_forward_saved(dev[0], dev[1], dev[2], dev[4], dev[5], st)
    g = ops.stable_backward_saved(dev[0], dev[1], dev[2], dev[3], s)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    c = lambda t: t.float().cpu()
    return dict(O=c(O), dQ=c(g[0]), dK=c(g[1]), dV=c(g[2]), top_idx=c(s.top_idx).long(),
                top_val=c(s.top_val), tau=c(s.tau), weights=c(s.weights))


@pytest.mark.parametrize("name", list(CASES))
def test_stable_operator(cuda, name):
    dt, d, alpha, sc, k, causal, sigma = CASES[name]
    B, H, N = 1, 2, 320
    Q, K, V, dO, Qi, Ki = make_inputs(B, H, N, N, d, seed=71, sigma=sigma, dtype=dt)
    got = engine(Q, K, V, dO, Qi, Ki, alpha, sc, k, causal, cuda)
    f = lambda x: x.float().reshape(B * H, N, d).numpy()
    cfg = orc.Config(B * H, N, N, d, 128, 128, k, alpha, sc, causal)
    ref = orc.stable_forward(cfg, f(Q), f(K), f(V), Qi.numpy(), Ki.numpy())
    # the kept keys are the reference's (bit-exact); the clamped scores
    # exactly for fp32 (same FMA chain), within fp32 summation error on the
    # tensor cores
    assert np.array_equal(got["top_idx"].numpy().reshape(ref["topi"].shape), ref["topi"])
    tv = got["top_val"].numpy().reshape(ref["topv"].shape)
    if dt == torch.float32:
        assert np.array_equal(tv, ref["topv"])
    else:
        assert np.abs(tv - ref["topv"]).max() <= 1e-4
    assert_close(f"{name} O", got["O"].numpy().reshape(ref["O"].shape), ref["O"], OUT_ATOL[dt])
    # gradient: float64 autograd through the same algorithm
    r = lambda t: t.double().reshape(B * H, N, d)
    q, kk, v = (r(t).requires_grad_() for t in (Q, K, V))
    O64, _, idx64 = stable_attention_f64(q, kk, v, Qi.long(), Ki.long(), alpha, sc, k, causal)
    assert torch.equal(idx64, got["top_idx"].reshape(idx64.shape))
    (O64 * r(dO)).sum().backward()
    tol = 1e-4 if dt == torch.float32 else 1e-3
    for key, g in (("dQ", q.grad), ("dK", kk.grad), ("dV", v.grad)):
        err = float((got[key].double().reshape(g.shape) - g).abs().max())
        assert err <= tol, f"{name} {key}: {err:.3g} > {tol}"


def test_notebook_signature_functions(cuda):
    import splash_attention as sa
    Q, K, V, dO, Qi, Ki = (x.to(cuda) for x in make_inputs(1, 2, 128, 128, 64, seed=72))
    O = sa.stable_forward(Q, K, V, Qi, Ki, 0.125, 1.5)
    dQ, dK, dV = sa.stable_backward(Q, K, V, Qi, Ki, 0.125, 1.5, dO)
    assert O.shape == Q.shape and dQ.shape == Q.shape and dK.shape == K.shape
    q, k, v = (x.clone().requires_grad_() for x in (Q, K, V))
    out = sa.stable_attention(q, k, v, Qi, Ki, alpha=1.5, sm_scale=0.125)
    out.backward(dO)
    torch.cuda.synchronize()
    assert torch.equal(out, O)
    for a, b in ((q.grad, dQ), (v.grad, dV)):
        assert torch.allclose(a, b, atol=1e-6)
