"""The registered PyTorch operators (csrc/torch_ops.cpp, _torch_ops.so):
schemas, Meta kernels and tracing, without a GPU.  They replace the
reference's pybind binding (source/adasplashattention.cu:702-705)."""
import pytest
import torch

import splash_attention as sa
from torch.fx.experimental.proxy_tensor import make_fx


def meta(*shape, dtype=torch.bfloat16):
    return torch.empty(*shape, dtype=dtype, device="meta")


def test_schemas_are_registered():
    f = str(torch.ops.splash_attention.forward.default._schema)
    b = str(torch.ops.splash_attention.backward.default._schema)
    assert f.startswith("splash_attention::forward(Tensor Q, Tensor K, Tensor V, Tensor? Q_idx")
    assert "-> (Tensor, Tensor, Tensor)" in b


@pytest.mark.parametrize("B,H,NQ,NK,d,out_dtype", [(2, 4, 300, 300, 128, None),
                                                  (1, 3, 130, 257, 64, torch.float32)])
def test_meta_shapes(B, H, NQ, NK, d, out_dtype):
    q, k = meta(B, H, NQ, d), meta(B, H, NK, d)
    qi = torch.arange(NQ, dtype=torch.int32, device="meta")
    ki = torch.arange(NK, dtype=torch.int32, device="meta")
    cfg = sa._op_config(q, sa.Settings(out_dtype=out_dtype))
    O, O32, tau, M, ptr, idx, rown = torch.ops.splash_attention.forward(
        q, k, k, qi.expand(B * H, NQ).contiguous(), ki.expand(B * H, NK).contiguous(), *cfg, True, True)
    nqb, nkb = -(-NQ // 128), -(-NK // 128)
    assert O.shape == (B, H, NQ, d) and O.dtype == (out_dtype or torch.bfloat16)
    assert O32.numel() == (0 if out_dtype == torch.float32 else B * H * NQ * d)
    assert tau.shape == rown.shape == (B * H, NQ) and M.shape == (B * H, nqb, nkb)
    assert ptr.shape == (B * H, nqb + 1) and idx.shape == (B * H, nqb * nkb)
    dQ, dK, dV = torch.ops.splash_attention.backward(q, k, k, None, None, O32, tau, M, ptr, idx,
                                                     rown, meta(B, H, NQ, d), *cfg)
    assert dQ.shape == q.shape and dK.shape == dV.shape == k.shape


def test_traces_to_one_operator_call():
    def f(q, k, v, i):
        return sa.splash_attention(q, k, v, i, i)
    q = meta(1, 2, 256, 128)
    g = make_fx(f, tracing_mode="fake")(q, q, q, torch.arange(256, dtype=torch.int32, device="meta"))
    calls = [n for n in g.graph.nodes if n.op == "call_function" and "splash_attention" in str(n.target)]
    assert len(calls) == 1


def test_autograd_is_attached():
    q = meta(1, 1, 128, 64).requires_grad_()
    out = sa.splash_attention(q, q, q, torch.arange(128, device="meta"), torch.arange(128, device="meta"))
    assert out.requires_grad and out.grad_fn is not None
