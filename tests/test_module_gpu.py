"""The drop-in Python surface: AdaptiveSplashAttention + autograd, and the
reference-signature forward/backward functions."""
import numpy as np
import pytest
import torch

from helpers import make_inputs, oracle_run, assert_close

pytestmark = pytest.mark.gpu


def test_readme_example_shapes_and_int64_indices(cuda):
    from splash_attention import AdaptiveSplashAttention
    B, H, N, d = 2, 8, 1024, 64
    attn = AdaptiveSplashAttention(head_dim=64, alpha=1.5, k_keep=8, adaptive_threshold=True,
                                   sm_scale=0.125)
    Q, K, V = (torch.randn(B, H, N, d, device=cuda) for _ in range(3))
    idx = torch.arange(N, device=cuda).expand(B * H, N).contiguous()   # int64, as README
    out = attn(Q, K, V, idx, idx)
    assert out.shape == Q.shape and out.dtype == Q.dtype and torch.isfinite(out).all()


def test_autograd_matches_oracle(cuda):
    from splash_attention import AdaptiveSplashAttention
    Q, K, V, dO, Qi, Ki = make_inputs(1, 2, 256, 256, 64, seed=21)
    attn = AdaptiveSplashAttention(64, alpha=1.5, k_keep=8, sm_scale=0.125, block_m=64, block_n=64)
    q, k, v = (x.to(cuda).requires_grad_() for x in (Q, K, V))
    out = attn(q, k, v, Qi.to(cuda), Ki.to(cuda))
    out.backward(dO.to(cuda))
    ref = oracle_run(Q, K, V, dO, Qi, Ki, 64, 64, 8, 1.5, 0.125)
    f = lambda t: t.detach().cpu().numpy().reshape(2, 256, 64)
    assert_close("O", f(out), ref["O"], 1e-5)
    assert_close("dQ", f(q.grad), ref["dQ"], 1e-5)
    assert_close("dK", f(k.grad), ref["dK"], 1e-5)
    assert_close("dV", f(v.grad), ref["dV"], 1e-5)


def test_reference_signature_functions(cuda):
    import splash_attention as sa
    Q, K, V, dO, Qi, Ki = make_inputs(1, 2, 256, 256, 64, seed=22)
    dev = [x.to(cuda) for x in (Q, K, V, Qi, Ki)]
    O = sa.forward(*dev, 0.125, 1.5)
    dQ, dK, dV = sa.backward(*dev, 0.125, 1.5, dO.to(cuda))
    # reference defaults BLOCK_M=32, BLOCK_N=64, K_KEEP=8 (:8-19)
    ref = oracle_run(Q, K, V, dO, Qi, Ki, 32, 64, 8, 1.5, 0.125)
    f = lambda t: t.cpu().numpy().reshape(2, 256, 64)
    assert_close("O", f(O), ref["O"], 1e-5)
    for name, g in (("dQ", dQ), ("dK", dK), ("dV", dV)):
        assert_close(name, f(g), ref[name], 1e-5)


def test_errors(cuda):
    from splash_attention import AdaptiveSplashAttention, splash_attention
    with pytest.raises(ValueError):
        AdaptiveSplashAttention(64, adaptive_threshold=False)
    q = torch.randn(1, 1, 64, 64)
    with pytest.raises(RuntimeError):
        splash_attention(q, q, q, torch.arange(64), torch.arange(64))   # CPU tensors
    qc = q.to(cuda)
    with pytest.raises(RuntimeError):
        splash_attention(qc, qc, qc, torch.arange(64), torch.arange(64), k_keep=40)
    with pytest.raises(TypeError):
        splash_attention(qc.half(), qc.half(), qc.half(), torch.arange(64), torch.arange(64))


def test_scrub_semantics(cuda):
    from splash_attention import ops
    x = torch.tensor([1.0, float("nan"), 250.0, -3.0], device=cuda)
    ops.scrub_(x)
    assert x.tolist() == [1.0, 0.0, 250.0, -3.0]
    x = torch.tensor([1.0, float("inf"), 250.0, float("nan")], device=cuda)
    ops.scrub_(x)
    assert x.tolist() == [1.0, 100.0, 100.0, 0.0]


def test_empty_sequences(cuda):
    from splash_attention import splash_attention
    q = torch.randn(1, 2, 0, 64, device=cuda)
    k = torch.randn(1, 2, 16, 64, device=cuda)
    out = splash_attention(q, k, k, torch.arange(0), torch.arange(16), block_m=32, block_n=32)
    assert out.shape == (1, 2, 0, 64)
