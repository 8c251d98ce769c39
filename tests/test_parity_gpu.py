"""Engine vs oracle parity on seeded inputs, through the C ABI (libasa.so)."""
import numpy as np
import pytest
import torch

from helpers import (make_inputs, oracle_run, assert_tau, assert_close, csr_equal, OUT_ATOL,
                     INT32_MAX)

pytestmark = pytest.mark.gpu

# name: B, H, NQ, NK, d, BM, BN, k_keep, alpha, sm_scale, causal, sigma, dtype, qoff, centroids, backend
CASES = {
    "c1_fp32": (1, 2, 256, 256, 64, 64, 64, 8, 1.5, 0.125, True, 1.0, torch.float32, 0, 0, "auto"),
    "c2s_fp32": (1, 2, 512, 512, 64, 32, 64, 8, 1.5, 0.125, True, 1.0, torch.float32, 0, 0, "auto"),
    "d128_fp32": (1, 2, 256, 256, 128, 32, 32, 8, 1.5, 128 ** -0.5, True, 1.0, torch.float32, 0, 0, "auto"),
    "alpha2_fp32": (1, 2, 256, 256, 64, 32, 64, 8, 2.0, 0.125, True, 1.0, torch.float32, 0, 0, "auto"),
    "alpha125_fp32": (1, 2, 256, 256, 64, 32, 64, 8, 1.25, 0.125, True, 1.0, torch.float32, 0, 0, "auto"),
    "alpha13_fp32": (1, 2, 256, 256, 64, 32, 64, 8, 1.3, 0.125, True, 1.0, torch.float32, 0, 0, "auto"),
    "noncausal_k16": (1, 2, 256, 256, 64, 32, 64, 16, 1.5, 0.125, False, 2.0, torch.float32, 0, 0, "auto"),
    "ragged": (1, 2, 200, 300, 64, 32, 64, 8, 1.5, 0.125, True, 1.0, torch.float32, 100, 0, "auto"),
    "saturated": (1, 1, 256, 256, 64, 32, 64, 8, 1.5, 0.125, True, 3.0, torch.float32, 0, 0, "auto"),
    "odd_d48": (1, 3, 130, 130, 48, 64, 32, 4, 1.5, 0.15, True, 1.0, torch.float32, 0, 0, "auto"),
    "noncausal_ragged": (1, 2, 200, 200, 64, 32, 64, 8, 1.5, 0.125, False, 1.0, torch.float32, 0, 0, "auto"),
    "k32": (1, 1, 256, 256, 64, 64, 64, 32, 1.5, 0.125, True, 1.0, torch.float32, 0, 0, "auto"),
    "bf16_c3s_simt": (1, 2, 512, 512, 128, 128, 128, 8, 1.5, 128 ** -0.5, True, 1.0, torch.bfloat16, 0, 0, "simt"),
    "bf16_c3s": (1, 2, 512, 512, 128, 128, 128, 8, 1.5, 128 ** -0.5, True, 1.0, torch.bfloat16, 0, 0, "auto"),
    "bf16_c5s": (2, 1, 512, 512, 64, 128, 128, 16, 1.25, 0.125, False, 2.0, torch.bfloat16, 0, 0, "auto"),
    "bf16_c4s": (1, 2, 1024, 1024, 128, 128, 128, 8, 2.0, 128 ** -0.5, True, 1.0, torch.bfloat16, 0, 64, "auto"),
    # tensor-core path: ragged NQ != NK with shifted query positions, ragged
    # non-causal keys, many key blocks per row, scores saturating the ±10 clamp
    "bf16_ragged": (1, 2, 200, 300, 128, 128, 128, 8, 1.5, 128 ** -0.5, True, 1.0, torch.bfloat16, 100, 0, "auto"),
    "bf16_noncausal_ragged": (1, 2, 200, 330, 64, 128, 128, 16, 1.5, 0.125, False, 1.0, torch.bfloat16, 0, 0, "auto"),
    "bf16_n2048": (1, 2, 2048, 2048, 128, 128, 128, 8, 1.5, 128 ** -0.5, True, 1.0, torch.bfloat16, 0, 0, "auto"),
    "bf16_saturated": (1, 1, 512, 512, 128, 128, 128, 8, 1.5, 0.3, True, 3.0, torch.bfloat16, 0, 0, "auto"),
}


def run_engine(Q, K, V, dO, Qi, Ki, BM, BN, kk, alpha, sc, causal, backend, precision="split",
               ref_tile_load=True):
    from splash_attention import ops
    st = ops.Settings(alpha=alpha, sm_scale=sc, k_keep=kk, block_m=BM, block_n=BN, causal=causal,
                      backend=backend, precision=precision, out_dtype=torch.float32,
                      ref_tile_load=ref_tile_load)
    dev = "cuda"
    Qd, Kd, Vd, dOd = (x.to(dev) for x in (Q, K, V, dO))
    O, s = ops.forward_saved(Qd, Kd, Vd, Qi.to(dev), Ki.to(dev), st)
    dQ, dK, dV = ops.backward_saved(Qd, Kd, Vd, dOd, s)
    torch.cuda.synchronize()
    assert ops.device_error() == 0, "a kernel's bounded wait ran out"
    c = lambda x: x.cpu().numpy()
    B, H = Q.shape[:2]
    f = lambda x: c(x).reshape(B * H, x.shape[2], x.shape[3])
    return dict(O=f(O), dQ=f(dQ), dK=f(dK), dV=f(dV), tau=c(s.tau), M=c(s.M), ptr=c(s.csr_ptr),
                idx=c(s.csr_idx), rownorm=c(s.rownorm), backend=ops.resolved_backend(s.params[0]))


@pytest.mark.parametrize("name", list(CASES))
def test_engine_matches_oracle(cuda, name):
    B, H, NQ, NK, d, BM, BN, kk, alpha, sc, causal, sigma, dt, qoff, cent, backend = CASES[name]
    Q, K, V, dO, Qi, Ki = make_inputs(B, H, NQ, NK, d, seed=11, sigma=sigma, dtype=dt, qoff=qoff,
                                      centroids=cent)
    ref = oracle_run(Q, K, V, dO, Qi, Ki, BM, BN, kk, alpha, sc, causal)
    got = run_engine(Q, K, V, dO, Qi, Ki, BM, BN, kk, alpha, sc, causal, backend)
    assert np.array_equal(got["M"], ref["M"]), "block mask differs"
    csr_equal(got["ptr"], got["idx"], ref["ptr"], ref["idx"])
    assert_tau(got["tau"], ref["tau"], tensor_core=got["backend"] == "tc")
    for k in ("O", "dQ", "dK", "dV"):
        assert_close(k, got[k], ref[k], OUT_ATOL[dt])


def test_noncausal_equals_int32max_positions(cuda):
    Q, K, V, dO, Qi, Ki = make_inputs(1, 2, 256, 256, 64, seed=2)
    a = run_engine(Q, K, V, dO, Qi, Ki, 32, 64, 8, 1.5, 0.125, False, "auto")
    b = run_engine(Q, K, V, dO, torch.full_like(Qi, INT32_MAX), Ki, 32, 64, 8, 1.5, 0.125, True,
                   "auto")
    for k in a:
        if k != "backend":
            assert np.array_equal(a[k], b[k]), k


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_backward_is_deterministic(cuda, dt):
    Q, K, V, dO, Qi, Ki = make_inputs(1, 2, 512, 512, 128, seed=4, dtype=dt)
    a = run_engine(Q, K, V, dO, Qi, Ki, 128, 128, 8, 1.5, 0.09, True, "auto")
    b = run_engine(Q, K, V, dO, Qi, Ki, 128, 128, 8, 1.5, 0.09, True, "auto")
    for k in ("dQ", "dK", "dV", "O", "tau", "M"):
        assert np.array_equal(a[k], b[k]), k


@pytest.mark.parametrize("dt,BM,BN,d", [(torch.float32, 32, 64, 64), (torch.bfloat16, 128, 128, 128)])
def test_full_rows_mode_matches_oracle(cuda, dt, BM, BN, d):
    # ref_tile_load=False: every visible key is read in full
    Q, K, V, dO, Qi, Ki = make_inputs(1, 2, 384, 384, d, seed=13, dtype=dt)
    ref = oracle_run(Q, K, V, dO, Qi, Ki, BM, BN, 8, 1.5, d ** -0.5, True, ref_tile_load=False)
    got = run_engine(Q, K, V, dO, Qi, Ki, BM, BN, 8, 1.5, d ** -0.5, True, "auto",
                     ref_tile_load=False)
    assert np.array_equal(got["M"], ref["M"])
    assert_tau(got["tau"], ref["tau"], tensor_core=got["backend"] == "tc")
    for k in ("O", "dQ", "dK", "dV"):
        assert_close(k, got[k], ref[k], OUT_ATOL[dt])


def test_many_items_match_head_chunks(cuda):
    # more (head, query block) items than SMs: the persistent forward walks
    # several items per CTA; each head must equal the same head computed in a
    # call small enough for one item per CTA (the kernels are deterministic)
    Q, K, V, dO, Qi, Ki = make_inputs(1, 24, 1024, 1024, 128, seed=5, dtype=torch.bfloat16)
    full = run_engine(Q, K, V, dO, Qi, Ki, 128, 128, 8, 1.5, 128 ** -0.5, True, "auto")
    for h0 in range(0, 24, 6):
        sl = slice(h0, h0 + 6)
        part = run_engine(Q[:, sl], K[:, sl], V[:, sl], dO[:, sl], Qi[sl], Ki[sl], 128, 128, 8, 1.5,
                          128 ** -0.5, True, "auto")
        for k in ("O", "dQ", "dK", "dV", "tau", "rownorm"):
            assert np.array_equal(full[k][sl], part[k]), (k, h0)
