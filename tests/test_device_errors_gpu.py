"""Device-side timeouts reach the host: the library's wait probe makes one
bounded wait give up (a barrier phase nothing completes), the C ABI reports
ASA_ERR_DEVICE_TIMEOUT, and the Python surface raises RuntimeError on the
next call.  No GPU fault is involved: the probe's kernel returns on its own
with nothing in flight (reference behaviour replaced: CUDA_CHECK /
TORCH_CHECK after a synchronising launch, source/adasplashattention.cu:24-27)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wait_probe_sets_timeout_code(cuda):
    from splash_attention import ops, _lib as L
    assert ops.device_error() == 0
    ops.wait_probe(1000)
    assert ops.device_error() == L.ASA_ERR_DEVICE_TIMEOUT
    assert ops.device_error() == 0          # read-and-clear


def test_python_surface_raises_after_a_timeout(cuda):
    from splash_attention import ops, splash_attention, _lib as L
    q = torch.randn(1, 1, 256, 64, device=cuda)
    idx = torch.arange(256, device=cuda)
    with torch.no_grad():
        splash_attention(q, q, q, idx, idx, block_m=64, block_n=64)
    torch.cuda.synchronize()
    ops.wait_probe(1000)
    with torch.no_grad():   # enqueues the asynchronous read of the error word
        splash_attention(q, q, q, idx, idx, block_m=64, block_n=64)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match=r"timed out \(asa_status 5\)"):
        with torch.no_grad():
            splash_attention(q, q, q, idx, idx, block_m=64, block_n=64)
    assert ops.device_error() == 0          # the raise cleared the word
    with torch.no_grad():                   # and the context is still usable
        out = splash_attention(q, q, q, idx, idx, block_m=64, block_n=64)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
