"""Engine vs the reference's own CUDA kernels: the golden vectors in
tests/golden/ (made by tests/golden/make_golden.py on a B200) against the
engine's output on the same seeded inputs, through the C ABI."""
import os

import numpy as np
import pytest
import torch

import cases
from helpers import TAU_RTOL, TAU_ATOL

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.mark.parametrize("name", list(cases.CASES))
def test_engine_matches_reference_kernels(cuda, name):
    from splash_attention import ops
    g = dict(np.load(os.path.join(GOLD, f"{name}.npz")))
    s = cases.spec(name)
    Q, K, V, dO, Qi, Ki = cases.make_inputs(name)
    st = ops.Settings(alpha=s["alpha"], sm_scale=s["sm_scale"], k_keep=s["k_keep"],
                      block_m=s["BM"], block_n=s["BN"], causal=True, out_dtype=torch.float32)
    dev = [x.to(cuda) for x in (Q, K, V)]
    O, sv = ops.forward_saved(*dev, Qi.to(cuda), Ki.to(cuda), st)
    dQ, dK, dV = ops.backward_saved(*dev, dO.to(cuda), sv)
    BH, NQ, NK, d = s["B"] * s["H"], s["NQ"], s["NK"], s["d"]
    c = lambda t: t.cpu().numpy()
    r = dict(tau=c(sv.tau), M=c(sv.M), ptr=c(sv.csr_ptr), idx=c(sv.csr_idx),
             O=c(O).reshape(BH, NQ, d), dQ=c(dQ).reshape(BH, NQ, d),
             dK=c(dK).reshape(BH, NK, d), dV=c(dV).reshape(BH, NK, d))
    # the reference's last partial query block reads stale shared memory
    # (its threads past NQ exit before staging): compare complete blocks only
    nfb = NQ // s["BM"]
    full = nfb * s["BM"]
    partial = full != NQ
    assert np.array_equal(r["M"][:, :nfb], g["M"][:, :nfb]), "block mask differs"
    assert np.array_equal(r["ptr"][:, :nfb + 1], g["ptr"][:, :nfb + 1])
    for b in range(BH):
        n = r["ptr"][b, nfb]
        assert np.array_equal(r["idx"][b, :n], g["idx"][b, :n])
    err = np.abs(r["tau"][:, :full] - g["tau"][:, :full]) - (
        TAU_ATOL + TAU_RTOL * np.abs(g["tau"][:, :full]))
    assert (err <= 0).all(), f"τ: worst excess {err.max():.3g}"
    for k in ("O", "dQ") + (() if partial else ("dK", "dV")):
        gk = g[k].reshape(r[k].shape)
        rk = r[k]
        if k in ("O", "dQ"):
            gk, rk = gk[:, :full], rk[:, :full]
        # α with non-integral exponents (1.3) runs powf, whose results the
        # engine's kernels and the reference's reach in different operation
        # orders: there the 1e-5 bound is scaled by max(1, max|ref|)
        scale = max(1.0, np.abs(gk).max()) if s["alpha"] not in (1.25, 1.5, 2.0) else 1.0
        e = np.abs(rk - gk).max()
        assert e <= 1e-5 * scale, f"{k}: max-abs {e:.3g} > {1e-5 * scale:.3g}"
