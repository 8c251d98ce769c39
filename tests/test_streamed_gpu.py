"""forward_backward_host: a host-resident batch processed in head chunks
with the copies overlapped; every head's result must equal the device
API's (the kernels are deterministic and heads are independent)."""
import pytest
import torch

from helpers import make_inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("causal,chunk", [(True, 4), (False, 5), (True, 64), (True, None), (False, [1, 3, 2])])
def test_streamed_matches_device_api(cuda, causal, chunk):
    import splash_attention as sa
    from splash_attention import ops
    Q, K, V, dO, Qi, Ki = make_inputs(2, 3, 384, 384, 128, seed=21, dtype=torch.bfloat16)
    st = dict(alpha=1.5, sm_scale=128 ** -0.5, k_keep=8, causal=causal)
    got = sa.forward_backward_host(*(x.pin_memory() for x in (Q, K, V, dO)), Qi, Ki,
                                   heads_per_chunk=chunk, **st)
    dev = [x.to(cuda) for x in (Q, K, V, dO)]
    O, saved = ops.forward_saved(dev[0], dev[1], dev[2], Qi.to(cuda), Ki.to(cuda), ops.Settings(**st))
    grads = ops.backward_saved(dev[0], dev[1], dev[2], dev[3], saved)
    torch.cuda.synchronize()
    for name, g, w in zip(("O", "dQ", "dK", "dV"), got, (O,) + tuple(grads)):
        assert torch.equal(g, w.cpu()), name


def test_streamed_rejects_bad_chunk_sizes(cuda):
    import splash_attention as sa
    Q, K, V, dO, Qi, Ki = make_inputs(1, 2, 128, 128, 64, seed=3, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="sum to B\\*H"):
        sa.forward_backward_host(*(x.pin_memory() for x in (Q, K, V, dO)), Qi, Ki,
                                 heads_per_chunk=[1, 2], alpha=1.5, k_keep=8)
