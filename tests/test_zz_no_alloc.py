"""The allocation-free τ / block-mask entry point, asa_tau_mask_noalloc.

It exists for callers that cannot allocate device memory when they need
the mask -- a plugin inside a framework whose allocator forbids cudaMalloc,
or an embedded runtime that owns all device memory up front -- and takes
its scratch from a fixed device array inside libasa.so.  These tests call
it through the C ABI and compare it with asa_tau_mask, which takes a caller
workspace.  The file is named to be collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import make_inputs
from splash_attention import _lib as L

pytestmark = pytest.mark.gpu


def _params(B, H, N, d, causal=True):
    p = L.Params()
    L.lib().asa_params_default(ctypes.byref(p))
    p.B, p.H, p.NQ, p.NK, p.d = B, H, N, N, d
    p.sm_scale = d ** -0.5
    p.causal = 1 if causal else 0
    return p


def _outputs(p, dev):
    BH = p.B * p.H
    nqb, nkb = -(-p.NQ // p.block_m), -(-p.NK // p.block_n)
    return (torch.full((BH, p.NQ), float("nan"), device=dev),
            torch.full((BH, nqb, nkb), 7, device=dev, dtype=torch.uint8),
            torch.full((BH, nqb + 1), -1, device=dev, dtype=torch.int32),
            torch.full((BH, nqb * nkb), -1, device=dev, dtype=torch.int32))


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _run(fn_noalloc, p, Q, K, Qi, Ki, dev):
    tau, M, ptr, idx = _outputs(p, dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if fn_noalloc:
        rc = L.lib().asa_tau_mask_noalloc(ctypes.byref(p), _ptr(Q), _ptr(K), _ptr(Qi), _ptr(Ki),
                                          _ptr(tau), _ptr(M), _ptr(ptr), _ptr(idx), stream)
    else:
        f, b = ctypes.c_size_t(), ctypes.c_size_t()
        L.check(L.lib().asa_workspace_bytes(ctypes.byref(p), ctypes.byref(f), ctypes.byref(b)), "ws")
        ws = torch.empty(f.value, device=dev, dtype=torch.uint8)
        rc = L.lib().asa_tau_mask(ctypes.byref(p), _ptr(Q), _ptr(K), _ptr(Qi), _ptr(Ki), _ptr(tau),
                                  _ptr(M), _ptr(ptr), _ptr(idx), _ptr(ws), f.value, stream)
    L.check(rc, "tau_mask")
    torch.cuda.synchronize()
    return [t.cpu().numpy() for t in (tau, M, ptr, idx)]


@pytest.mark.parametrize("dtype,causal", [(torch.bfloat16, True), (torch.bfloat16, False),
                                          (torch.float32, True)])
def test_noalloc_matches_workspace_entry_point(cuda, dtype, causal):
    # bf16 at d=128 runs the tcgen05 kernels, whose per-block index bounds
    # live in the scratch; fp32 runs the CUDA-core kernels.
    p = _params(1, 2, 512, 128, causal)
    p.in_dtype = L.DTYPE_F32 if dtype == torch.float32 else L.DTYPE_BF16
    ref_inputs = make_inputs(1, 2, 512, 512, 128, seed=31, dtype=dtype)
    Q, K, _, _, Qi, Ki = (x.to(cuda) for x in ref_inputs)
    want = _run(False, p, Q, K, Qi, Ki, cuda)
    # two calls in a row: the second sees the first call's leftovers
    for call in range(2):
        got = _run(True, p, Q, K, Qi, Ki, cuda)
        # same kernels on the same inputs: every output bit-identical
        for g, w, name in zip(got, want, ("tau", "M", "csr_ptr", "csr_idx")):
            assert np.array_equal(g, w), f"call {call}: {name} differs"


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda):
    # 2*BH*(nQB+nKB) int32 bounds = 4096*2*512*4 bytes, far above 1 MiB
    p = _params(64, 64, 32768, 128)
    rc = L.lib().asa_tau_mask_noalloc(ctypes.byref(p), None, None, None, None, None, None, None,
                                      None, None)
    assert rc == L.ASA_ERR_WORKSPACE
    assert L.NOALLOC_SCRATCH_BYTES == 1 << 20
