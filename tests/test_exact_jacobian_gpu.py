"""The opt-in modes against float64 torch autograd (tests/entmax_f64.py):

* tau_mode="exact" + grad_mode="jacobian": exact α-entmax attention (τ over
  every visible key, Σp = 1) and its exact gradient; the block mask must
  contain every tile holding a positive weight ("tile max vs τ").
* grad_mode="jacobian" with the reference's top-k τ: the gradient of the
  output with τ moving so that each row's mass Σp stays at its value, over
  the reference mask's active tiles.

Tolerances: bf16 inputs 1e-3 max-abs (fp32 accumulation on the tensor
cores); fp32 inputs 1e-4 -- these compare the engine's fp32 arithmetic with
float64 mathematics, not with an fp32 reference whose rounding it follows.
τ within 1e-5 relative (+1e-6).
"""
import numpy as np
import pytest
import torch

from entmax_f64 import entmax_attention
from helpers import make_inputs

pytestmark = pytest.mark.gpu

ATOL = {torch.bfloat16: 1e-3, torch.float32: 1e-4}


def run(Q, K, V, dO, Qi, Ki, st, cuda):
    from splash_attention import ops
    dev = [x.to(cuda) for x in (Q, K, V, dO, Qi, Ki)]
    O, s = ops.forward_saved(*dev[:3], dev[4], dev[5], st)
    grads = ops.backward_saved(*dev[:3], dev[3], s)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    f = lambda t: t.float().cpu().reshape(-1, t.shape[2], t.shape[3])
    return dict(O=f(O), dQ=f(grads[0]), dK=f(grads[1]), dV=f(grads[2]), tau=s.tau.cpu(),
                M=s.M.cpu(), rownorm=s.rownorm.cpu(), backend=ops.resolved_backend(s.params[0]))


def f64_grads(Q, K, V, dO, Qi, Ki, alpha, sc, causal, keys=None, mass=None):
    BH = Q.shape[0] * Q.shape[1]
    r = lambda t: t.double().reshape(BH, t.shape[2], t.shape[3])
    q, k, v = (r(t).requires_grad_() for t in (Q, K, V))
    O, tau = entmax_attention(q, k, v, Qi.long(), Ki.long(), alpha, sc, causal, keys=keys, mass=mass)
    (O * r(dO)).sum().backward()
    return dict(O=O.detach(), dQ=q.grad, dK=k.grad, dV=v.grad, tau=tau.detach())


def close(name, got, ref, atol):
    err = float((got.double() - ref).abs().max())
    assert err <= atol, f"{name}: max-abs {err:.3g} > {atol:.3g}"


CASES = {
    # name: dtype, d, BM, BN, alpha, sm_scale, causal
    "tc_d128_a15": (torch.bfloat16, 128, 128, 128, 1.5, 128 ** -0.5, True),
    "tc_d128_a2": (torch.bfloat16, 128, 128, 128, 2.0, 128 ** -0.5, True),
    "tc_d64_a125_noncausal": (torch.bfloat16, 64, 128, 128, 1.25, 0.125, False),
    "simt_fp32_a15": (torch.float32, 64, 64, 64, 1.5, 0.125, True),
    "simt_fp32_a2_noncausal": (torch.float32, 64, 32, 64, 2.0, 0.125, False),
}


@pytest.mark.parametrize("name", list(CASES))
def test_exact_tau_and_jacobian_match_float64_entmax(cuda, name):
    from splash_attention import ops
    dt, d, BM, BN, alpha, sc, causal = CASES[name]
    N = 384
    Q, K, V, dO, Qi, Ki = make_inputs(1, 2, N, N, d, seed=61, dtype=dt)
    st = ops.Settings(alpha=alpha, sm_scale=sc, block_m=BM, block_n=BN, causal=causal,
                      out_dtype=torch.float32, tau_mode="exact", grad_mode="jacobian")
    got = run(Q, K, V, dO, Qi, Ki, st, cuda)
    assert got["backend"] == ("tc" if dt == torch.bfloat16 else "simt")
    ref = f64_grads(Q, K, V, dO, Qi, Ki, alpha, sc, causal)
    tau_err = (got["tau"].double() - ref["tau"]).abs() - (1e-6 + 1e-5 * ref["tau"].abs())
    assert float(tau_err.max()) <= 0, f"τ: worst excess {float(tau_err.max()):.3g}"
    # every tile with a positive weight is in the mask
    am1 = alpha - 1
    s = torch.clamp(sc * torch.einsum("bqd,bkd->bqk", Q.double().reshape(2, N, d),
                                      K.double().reshape(2, N, d)), -10, 10)
    vis = (Ki[:, None, :] <= Qi[:, :, None]) if causal else torch.ones(2, N, N, dtype=torch.bool)
    pos = ((am1 * s - ref["tau"][..., None]) > 1e-9) & vis
    need = pos.reshape(2, N // BM, BM, N // BN, BN).any(-1).any(2)
    assert bool((got["M"].bool() | ~need).all()), "mask misses a tile with positive weight"
    for k in ("O", "dQ", "dK", "dV"):
        close(f"{name} {k}", got[k], ref[k], ATOL[dt])


@pytest.mark.parametrize("dt,d,BM,BN", [(torch.bfloat16, 128, 128, 128), (torch.float32, 64, 32, 64)])
def test_jacobian_with_reference_tau(cuda, dt, d, BM, BN):
    from splash_attention import ops
    N, alpha, sc = 384, 1.5, d ** -0.5
    Q, K, V, dO, Qi, Ki = make_inputs(1, 2, N, N, d, seed=62, dtype=dt)
    st = ops.Settings(alpha=alpha, sm_scale=sc, block_m=BM, block_n=BN, out_dtype=torch.float32,
                      ref_tile_load=False, grad_mode="jacobian")
    got = run(Q, K, V, dO, Qi, Ki, st, cuda)
    # the f64 objective: keys of the active tiles, row mass held at the value
    # the forward's τ gives (its τ solves Σp = mass)
    keys = got["M"].bool().repeat_interleave(BM, 1).repeat_interleave(BN, 2)[:, :N, :N]
    s = torch.clamp(sc * torch.einsum("bqd,bkd->bqk", Q.double().reshape(2, N, d),
                                      K.double().reshape(2, N, d)), -10, 10)
    vis = (Ki[:, None, :] <= Qi[:, :, None]) & keys
    p = torch.clamp((alpha - 1) * s - got["tau"].double()[..., None], min=0) ** (1 / (alpha - 1)) * vis
    ref = f64_grads(Q, K, V, dO, Qi, Ki, alpha, sc, True, keys=keys, mass=p.sum(-1))
    assert float((ref["tau"] - got["tau"].double()).abs().max()) < 1e-5
    for k in ("O", "dQ", "dK", "dV"):
        close(f"jacobian/reference-τ {k}", got[k], ref[k], ATOL[dt])
