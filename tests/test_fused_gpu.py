"""The fused forward (one kernel per query block: τ / mask, then the forward
over the block's active key blocks) against the separate launches
(k1_tau_mask -> k1_tau_solve -> tile lists -> k3_forward).

Both run the same phase code, the same τ solve on the same top-k values and
the same epilogue width, so every output must be bit-identical: O, O32, τ,
the block mask, the CSR and Σp.  The oracle parity of the default (fused)
path is covered by the other GPU parity tests; this file pins that the
fusion itself changes nothing, including on ragged shapes, saturated rows,
partial query blocks and empty query blocks; with k = 16 (served by the
separate launches) the request must fall back and still agree.
"""
import pytest
import torch

from helpers import make_inputs

pytestmark = pytest.mark.gpu

CASES = {
    # name: (B, H, NQ, NK, d, k, alpha, sigma, causal, qoff, centroids)
    "c3_like": (1, 2, 4096, 4096, 128, 8, 1.5, 1.0, True, 0, 0),
    "d64_k16": (1, 2, 2048, 2048, 64, 16, 1.5, 1.0, False, 0, 0),
    "k16_causal_d128": (2, 1, 1536, 1536, 128, 16, 2.0, 1.0, True, 0, 0),
    "ragged": (1, 3, 700, 1100, 128, 8, 1.25, 1.0, True, 400, 0),
    "saturated": (1, 2, 1024, 1024, 128, 8, 1.5, 8.0, True, 0, 0),
    "clusters": (1, 2, 2048, 2048, 128, 8, 2.0, 1.0, True, 0, 16),
    "alpha13": (1, 2, 1024, 1024, 64, 8, 1.3, 1.0, True, 0, 0),
    # odd query-block counts: the separate forward pairs query blocks per CTA
    "odd_blocks": (1, 2, 640, 640, 128, 8, 1.5, 1.0, True, 0, 0),
    "odd_partial": (2, 1, 300, 900, 64, 8, 2.0, 1.0, True, 600, 0),
    "odd_noncausal": (1, 2, 384, 1000, 128, 8, 1.5, 1.0, False, 0, 0),
    # queries whose positions precede every key: an empty first query block
    "empty_blocks": (1, 1, 512, 512, 128, 8, 1.5, 1.0, True, -200, 0),
}


def forward(dev, st):
    from splash_attention import ops
    Q, K, V, Qi, Ki = dev
    O, s = ops.forward_saved(Q, K, V, Qi, Ki, st, need_o32=True)
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    return O, s


@pytest.mark.parametrize("name", sorted(CASES))
def test_fused_forward_equals_separate_launches(name, cuda):
    from splash_attention import ops
    B, H, NQ, NK, d, k, alpha, sigma, causal, qoff, cent = CASES[name]
    Q, K, V, _, Qi, Ki = make_inputs(B, H, NQ, NK, d, seed=21, sigma=sigma, dtype=torch.bfloat16,
                                     causal=causal, qoff=qoff, centroids=cent)
    dev = [x.to(cuda) for x in (Q, K, V, Qi, Ki)]
    base = dict(alpha=alpha, k_keep=k, sm_scale=d ** -0.5, causal=causal, backend="tc")
    with ops.profile() as prof:
        Of, sf = forward(dev, ops.Settings(fused_forward=True, **base))
    # the fused kernel serves k <= 8; larger k runs the separate launches
    assert ("forward_fused" in prof.result) == (k <= 8)
    assert ("tau_mask" in prof.result) == (k > 8)
    with ops.profile() as prof:
        Os, ss = forward(dev, ops.Settings(fused_forward=False, **base))
    assert "forward_fused" not in prof.result and "tau_mask" in prof.result
    assert torch.equal(Of, Os)
    assert torch.equal(sf.O32, ss.O32)
    assert torch.equal(sf.tau, ss.tau)
    assert torch.equal(sf.M, ss.M)
    assert torch.equal(sf.rownorm, ss.rownorm)
    assert torch.equal(sf.csr_ptr, ss.csr_ptr)
    for bh in range(B * H):
        n = int(sf.csr_ptr[bh, -1])
        assert torch.equal(sf.csr_idx[bh, :n], ss.csr_idx[bh, :n])


def test_fused_forward_backward_matches(cuda):
    """The backward from the fused forward's saved state equals the one from
    the separate launches' (it reads τ, M, the CSR, Σp and O32)."""
    from splash_attention import ops
    Q, K, V, dO, Qi, Ki = make_inputs(1, 2, 2048, 2048, 128, seed=5, dtype=torch.bfloat16)
    dev = [x.to(cuda) for x in (Q, K, V, Qi, Ki)]
    dOd = dO.to(cuda)
    out = []
    for fused in (True, False):
        st = ops.Settings(fused_forward=fused, backend="tc")
        _, s = forward(dev, st)
        out.append(ops.backward_saved(dev[0], dev[1], dev[2], dOd, s))
    torch.cuda.synchronize()
    for a, b in zip(*out):
        assert torch.equal(a, b)


def test_fused_is_the_default_on_the_operator(cuda):
    import splash_attention as sa
    from splash_attention import ops
    Q, K, V, _, Qi, Ki = make_inputs(1, 1, 512, 512, 128, seed=3, dtype=torch.bfloat16)
    q, k, v, qi, ki = (x.to(cuda) for x in (Q, K, V, Qi, Ki))
    with ops.profile() as prof:
        O1 = sa.splash_attention(q, k, v, qi, ki)
    assert "forward_fused" in prof.result
    O2 = sa.splash_attention(q, k, v, qi, ki, fused_forward=False)
    torch.cuda.synchronize()
    assert torch.equal(O1, O2)
