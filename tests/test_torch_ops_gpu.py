"""The registered operators on the GPU: identical results to the C-ABI path
(ops.forward_saved / backward_saved through ctypes), and PyTorch's own
operator checks (schema, fake tensors, autograd registration)."""
import numpy as np
import pytest
import torch

from helpers import make_inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt,BM,BN,d", [(torch.bfloat16, 128, 128, 128), (torch.float32, 32, 64, 64)])
def test_operator_equals_c_abi_path(cuda, dt, BM, BN, d):
    import splash_attention as sa
    from splash_attention import ops
    Q, K, V, dO, Qi, Ki = (x.to(cuda) for x in make_inputs(1, 2, 384, 384, d, seed=3, dtype=dt))
    q, k, v = (x.clone().requires_grad_() for x in (Q, K, V))
    out = sa.splash_attention(q, k, v, Qi, Ki, block_m=BM, block_n=BN)
    out.backward(dO)
    st = ops.Settings(block_m=BM, block_n=BN)
    O, s = ops.forward_saved(Q, K, V, Qi, Ki, st)
    dQ, dK, dV = ops.backward_saved(Q, K, V, dO, s)
    torch.cuda.synchronize()
    for a, b in ((out, O), (q.grad, dQ), (k.grad, dK), (v.grad, dV)):
        assert torch.equal(a, b.to(a.dtype))


def test_opcheck(cuda):
    import splash_attention as sa
    Q, K, V, dO, Qi, Ki = (x.to(cuda) for x in make_inputs(1, 2, 256, 256, 128, seed=4,
                                                          dtype=torch.bfloat16))
    args = (Q, K, V, Qi, Ki) + sa._op_config(Q, sa.Settings()) + (True, True)
    torch.library.opcheck(torch.ops.splash_attention.forward.default, args,
                          test_utils=("test_schema", "test_faketensor", "test_autograd_registration"))
