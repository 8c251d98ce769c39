"""Tensor-level operations over the C ABI: τ/mask, forward, backward.

All buffers are allocated here with torch (device memory and the current
stream are torch's); every computation runs in libasa.so's CUDA kernels.

Reference surface mirrored (mvideet/Adaptive-Splash-Attention,
source/adasplashattention.cu): ``forward(Q, K, V, Q_idx, K_idx, sm_scale,
alpha)`` (:537-609, :703) and ``backward(Q, K, V, Q_idx, K_idx, sm_scale,
alpha, dOut)`` (:611-700, :704).
"""
import ctypes
import math
from dataclasses import dataclass

import torch

from . import _lib as L


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _dtype_code(dt):
    if dt == torch.float32:
        return L.DTYPE_F32
    if dt == torch.bfloat16:
        return L.DTYPE_BF16
    raise TypeError(f"splash_attention: unsupported dtype {dt} (float32 or bfloat16)")


def _torch_dtype(code):
    return torch.float32 if code == L.DTYPE_F32 else torch.bfloat16


@dataclass
class Settings:
    """Per-call settings; the reference fixes most of these at compile time
    (BLOCK_M, BLOCK_N, K_KEEP: adasplashattention.cu:8-19)."""
    alpha: float = 1.5
    sm_scale: float = None
    k_keep: int = 8
    block_m: int = 128
    block_n: int = 128
    causal: bool = True
    backend: str = "auto"
    precision: str = "split"
    out_dtype: torch.dtype = None
    timeout_spins: int = 0
    # reproduce the reference's tile-load zeroing (include/asa.h ref_tile_load)
    ref_tile_load: bool = True
    # "reference": τ from the row's top-k (the reference); "exact": the exact
    # α-entmax threshold over all visible keys, mask = tiles with weight
    tau_mode: str = "reference"
    # "reference": the fixed-τ gradient; "jacobian": the α-entmax Jacobian
    grad_mode: str = "reference"
    # tcgen05 forward: one fused τ / mask + forward kernel (include/asa.h
    # fused_forward); False runs the separate launches
    fused_forward: bool = True


def make_params(Q, K, st: Settings):
    if Q.dim() != 4 or K.dim() != 4:
        raise ValueError("splash_attention: Q, K, V must be [B, H, N, d]")
    B, H, NQ, d = Q.shape
    NK = K.shape[2]
    if K.shape[0] != B or K.shape[1] != H or K.shape[3] != d:
        raise ValueError("splash_attention: K must be [B, H, NK, d] matching Q")
    p = L.Params()
    L.lib().asa_params_default(ctypes.byref(p))
    p.B, p.H, p.NQ, p.NK, p.d = B, H, NQ, NK, d
    p.block_m, p.block_n, p.k_keep = int(st.block_m), int(st.block_n), int(st.k_keep)
    p.alpha = float(st.alpha)
    p.sm_scale = float(st.sm_scale if st.sm_scale is not None else 1.0 / math.sqrt(d))
    p.causal = 1 if st.causal else 0
    p.in_dtype = _dtype_code(Q.dtype)
    p.out_dtype = _dtype_code(st.out_dtype if st.out_dtype is not None else Q.dtype)
    p.backend = L.BACKEND[st.backend]
    p.precision = L.PRECISION[st.precision]
    p.timeout_spins = int(st.timeout_spins)
    p.ref_tile_load = 1 if st.ref_tile_load else 0
    if st.tau_mode not in L.TAU_MODE or st.grad_mode not in L.GRAD_MODE:
        raise ValueError(f"splash_attention: tau_mode in {tuple(L.TAU_MODE)}, "
                         f"grad_mode in {tuple(L.GRAD_MODE)}")
    p.tau_mode = L.TAU_MODE[st.tau_mode]
    p.grad_mode = L.GRAD_MODE[st.grad_mode]
    p.fused_forward = 1 if st.fused_forward else 0
    return p


def resolved_backend(p):
    b = L.lib().asa_resolve_backend(ctypes.byref(p))
    if b < 0:
        L.check(-b, "asa_resolve_backend")
    return L.BACKEND_NAME[b]


def _workspace(p, device):
    fwd = ctypes.c_size_t()
    bwd = ctypes.c_size_t()
    L.check(L.lib().asa_workspace_bytes(ctypes.byref(p), ctypes.byref(fwd), ctypes.byref(bwd)),
            "asa_workspace_bytes")
    return fwd.value, bwd.value


def _index(idx, BH, N, device, name):
    """Position indices as contiguous int32 [B*H, N] (the reference requires
    int32 [B*H, N], :571-572; the README passes int64 arange, so it is cast)."""
    if idx is None:
        raise ValueError(f"splash_attention: {name} is required when causal=True")
    if not isinstance(idx, torch.Tensor):
        idx = torch.as_tensor(idx)
    idx = idx.to(device=device)
    if idx.dim() == 1:
        idx = idx.unsqueeze(0).expand(BH, N)
    idx = idx.reshape(BH, N)
    if idx.dtype != torch.int32:
        idx = idx.to(torch.int32)
    return idx.contiguous()


def _check_inputs(*ts):
    dev = ts[0].device
    if dev.type != "cuda":
        raise RuntimeError("splash_attention: tensors must be on a CUDA device")  # reference :543
    for t in ts:
        if t is not None and t.device != dev:
            raise RuntimeError("splash_attention: all tensors must be on the same device")


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class Saved:
    """What the forward hands the backward: τ, the block mask and its CSR,
    Σp per query and the fp32 output."""
    __slots__ = ("tau", "M", "csr_ptr", "csr_idx", "rownorm", "O32", "params")


def tau_mask(Q, K, Q_idx, K_idx, st: Settings):
    """τ [B*H, NQ] fp32, block mask M uint8 [B*H, nQB, nKB], CSR (ptr, idx)."""
    _check_inputs(Q, K)
    Q, K = Q.contiguous(), K.contiguous()
    p = make_params(Q, K, st)
    BH = p.B * p.H
    nQB = -(-p.NQ // p.block_m)
    nKB = -(-p.NK // p.block_n)
    dev = Q.device
    qi = _index(Q_idx, BH, p.NQ, dev, "Q_idx") if st.causal else None
    ki = _index(K_idx, BH, p.NK, dev, "K_idx") if st.causal else None
    tau = torch.empty(BH, p.NQ, device=dev, dtype=torch.float32)
    M = torch.empty(BH, nQB, nKB, device=dev, dtype=torch.uint8)
    ptr = torch.empty(BH, nQB + 1, device=dev, dtype=torch.int32)
    idx = torch.empty(BH, nQB * nKB, device=dev, dtype=torch.int32)
    fwd, _ = _workspace(p, dev)
    ws = torch.empty(fwd, device=dev, dtype=torch.uint8)
    L.check(L.lib().asa_tau_mask(ctypes.byref(p), _ptr(Q), _ptr(K), _ptr(qi), _ptr(ki), _ptr(tau),
                                 _ptr(M), _ptr(ptr), _ptr(idx), _ptr(ws), fwd, _stream()),
            "asa_tau_mask")
    return tau, M, ptr, idx


def forward_saved(Q, K, V, Q_idx, K_idx, st: Settings, need_o32=True):
    """Forward pass; returns (O, Saved)."""
    _check_inputs(Q, K, V)
    Q, K, V = Q.contiguous(), K.contiguous(), V.contiguous()
    if V.shape != K.shape or V.dtype != Q.dtype or K.dtype != Q.dtype:
        raise ValueError("splash_attention: V must match K in shape and Q in dtype")
    p = make_params(Q, K, st)
    BH = p.B * p.H
    nQB = -(-p.NQ // p.block_m)
    nKB = -(-p.NK // p.block_n)
    dev = Q.device
    qi = _index(Q_idx, BH, p.NQ, dev, "Q_idx") if st.causal else None
    ki = _index(K_idx, BH, p.NK, dev, "K_idx") if st.causal else None
    out_dt = _torch_dtype(p.out_dtype)
    O = torch.empty(p.B, p.H, p.NQ, p.d, device=dev, dtype=out_dt)
    if out_dt == torch.float32:
        O32 = O
    else:
        O32 = torch.empty(p.B, p.H, p.NQ, p.d, device=dev, dtype=torch.float32) if need_o32 else None
    s = Saved()
    s.tau = torch.empty(BH, p.NQ, device=dev, dtype=torch.float32)
    s.M = torch.empty(BH, nQB, nKB, device=dev, dtype=torch.uint8)
    s.csr_ptr = torch.empty(BH, nQB + 1, device=dev, dtype=torch.int32)
    s.csr_idx = torch.empty(BH, nQB * nKB, device=dev, dtype=torch.int32)
    s.rownorm = torch.empty(BH, p.NQ, device=dev, dtype=torch.float32)
    s.O32 = O32
    s.params = (p, qi, ki)
    fwd, _ = _workspace(p, dev)
    ws = torch.empty(fwd, device=dev, dtype=torch.uint8)
    check_device_errors(dev)
    L.check(L.lib().asa_forward(ctypes.byref(p), _ptr(Q), _ptr(K), _ptr(V), _ptr(qi), _ptr(ki),
                                _ptr(O), _ptr(O32), _ptr(s.tau), _ptr(s.M), _ptr(s.csr_ptr),
                                _ptr(s.csr_idx), _ptr(s.rownorm), _ptr(ws), fwd, _stream()),
            "asa_forward")
    if not need_o32:   # no backward will follow: read the error word now
        _poll_device_errors(dev)
    return O, s


def backward_saved(Q, K, V, dO, s: Saved):
    """Backward from a forward's Saved state; returns (dQ, dK, dV)."""
    p, qi, ki = s.params
    Q, K, V = Q.contiguous(), K.contiguous(), V.contiguous()
    dO = dO.to(Q.dtype).contiguous()
    dev = Q.device
    out_dt = _torch_dtype(p.out_dtype)
    dQ = torch.empty(Q.shape, device=dev, dtype=out_dt)
    dK = torch.empty(K.shape, device=dev, dtype=out_dt)
    dV = torch.empty(V.shape, device=dev, dtype=out_dt)
    _, bwd = _workspace(p, dev)
    ws = torch.empty(bwd, device=dev, dtype=torch.uint8)
    check_device_errors(dev)
    L.check(L.lib().asa_backward(ctypes.byref(p), _ptr(Q), _ptr(K), _ptr(V), _ptr(qi), _ptr(ki),
                                 _ptr(s.O32), _ptr(s.tau), _ptr(s.M), _ptr(s.csr_ptr),
                                 _ptr(s.csr_idx), _ptr(s.rownorm), _ptr(dO), _ptr(dQ), _ptr(dK),
                                 _ptr(dV), _ptr(ws), bwd, _stream()),
            "asa_backward")
    _poll_device_errors(dev)
    return dQ, dK, dV


def scrub_(x):
    """In-place device version of the reference's host scrub (:599-606)."""
    ws = torch.empty(16, device=x.device, dtype=torch.uint8)
    L.check(L.lib().asa_scrub(_dtype_code(x.dtype), _ptr(x), x.numel(), _ptr(ws), _stream()),
            "asa_scrub")
    return x


def device_error(device=None):
    """Read and clear the device error word (bounded waits that ran out).
    Synchronises the current stream."""
    code = ctypes.c_int()
    with torch.cuda.device(device):
        L.check(L.lib().asa_device_error(_stream(), ctypes.byref(code)), "asa_device_error")
    return code.value


# Per device: a pinned host int that receives asynchronous copies of the
# device error word after each backward (and each forward that saves nothing
# for a backward).  A copy that has landed with a non-zero value makes the
# next call raise -- the reference raises from CUDA_CHECK / TORCH_CHECK after
# its synchronising launches (:24-27); here no call synchronises, so the
# report comes one call later, or from device_error() at any time.
_err_words = {}


def _error_word(dev):
    w = _err_words.get(dev)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        _err_words[dev] = w
    return w


def check_device_errors(dev):
    """Raise AsaError(ASA_ERR_DEVICE_TIMEOUT) if an earlier asynchronous
    read of the device error word on `dev` saw a timed-out wait."""
    w = _err_words.get(dev)
    if w is not None and int(w[0]) != 0:
        code = int(w[0])
        w[0] = 0
        with torch.cuda.device(dev):
            device_error()          # clears the device word
        raise L.AsaError(code, "a previous splash_attention call on this device")


def _poll_device_errors(dev):
    w = _error_word(dev)
    code = ctypes.c_int.from_address(w.data_ptr())
    L.check(L.lib().asa_device_error_async(_stream(), ctypes.byref(code)),
            "asa_device_error_async")


def wait_probe(spins=1000):
    """Launch the library's device-timeout self-test on the current stream:
    a wait that nothing completes gives up after `spins` polls and records
    ASA_ERR_DEVICE_TIMEOUT in the device error word."""
    L.check(L.lib().asa_wait_probe(int(spins), _stream()), "asa_wait_probe")


class profile:
    """Context manager over asa_profile_begin/end: per-kernel-label device
    time (ms) and launch counts of everything the library launches inside
    the block on this thread.  ``.result`` maps label -> (total_ms, launches)."""

    def __enter__(self):
        L.check(L.lib().asa_profile_begin(1), "asa_profile_begin")
        self.result = {}
        return self

    def __exit__(self, *exc):
        L.check(L.lib().asa_profile_end(), "asa_profile_end")
        i = 0
        lab, ms, n = ctypes.c_char_p(), ctypes.c_double(), ctypes.c_int()
        while L.lib().asa_profile_get(i, ctypes.byref(lab), ctypes.byref(ms), ctypes.byref(n)) == 0:
            self.result[lab.value.decode()] = (ms.value, n.value)
            i += 1
        return False


def launch_count():
    return int(L.lib().asa_launch_count())


class StableSaved:
    """What the top-k-only operator's forward hands its backward."""
    __slots__ = ("top_val", "top_idx", "weights", "tau", "tau_coef", "params")


def stable_forward_saved(Q, K, V, Q_idx, K_idx, st: Settings):
    """The notebook's top-k-only ("stable") operator (asa_stable_forward);
    returns (O, StableSaved).  Q, K, V: [B, H, N, d]."""
    _check_inputs(Q, K, V)
    Q, K, V = Q.contiguous(), K.contiguous(), V.contiguous()
    if V.shape != K.shape or V.dtype != Q.dtype or K.dtype != Q.dtype:
        raise ValueError("stable_attention: V must match K in shape and Q in dtype")
    p = make_params(Q, K, st)
    BH = p.B * p.H
    dev = Q.device
    qi = _index(Q_idx, BH, p.NQ, dev, "Q_idx") if st.causal else None
    ki = _index(K_idx, BH, p.NK, dev, "K_idx") if st.causal else None
    O = torch.empty(p.B, p.H, p.NQ, p.d, device=dev, dtype=_torch_dtype(p.out_dtype))
    s = StableSaved()
    s.top_val = torch.empty(BH, p.NQ, p.k_keep, device=dev, dtype=torch.float32)
    s.top_idx = torch.empty(BH, p.NQ, p.k_keep, device=dev, dtype=torch.int32)
    s.weights = torch.empty(BH, p.NQ, p.k_keep, device=dev, dtype=torch.float32)
    s.tau = torch.empty(BH, p.NQ, device=dev, dtype=torch.float32)
    s.tau_coef = torch.empty(BH, p.NQ, device=dev, dtype=torch.float32)
    s.params = p
    fwd, bwd = ctypes.c_size_t(), ctypes.c_size_t()
    L.check(L.lib().asa_stable_workspace_bytes(ctypes.byref(p), ctypes.byref(fwd), ctypes.byref(bwd)),
            "asa_stable_workspace_bytes")
    ws = torch.empty(fwd.value, device=dev, dtype=torch.uint8)
    check_device_errors(dev)
    L.check(L.lib().asa_stable_forward(ctypes.byref(p), _ptr(Q), _ptr(K), _ptr(V), _ptr(qi), _ptr(ki),
                                       _ptr(O), _ptr(s.top_val), _ptr(s.top_idx), _ptr(s.weights),
                                       _ptr(s.tau), _ptr(s.tau_coef), _ptr(ws), fwd.value, _stream()),
            "asa_stable_forward")
    return O, s


def stable_backward_saved(Q, K, V, dO, s: StableSaved):
    """Gradient of the top-k-only operator (asa_stable_backward)."""
    p = s.params
    Q, K, V = Q.contiguous(), K.contiguous(), V.contiguous()
    dO = dO.to(Q.dtype).contiguous()
    dev = Q.device
    out_dt = _torch_dtype(p.out_dtype)
    dQ = torch.empty(Q.shape, device=dev, dtype=out_dt)
    dK = torch.empty(K.shape, device=dev, dtype=out_dt)
    dV = torch.empty(V.shape, device=dev, dtype=out_dt)
    fwd, bwd = ctypes.c_size_t(), ctypes.c_size_t()
    L.check(L.lib().asa_stable_workspace_bytes(ctypes.byref(p), ctypes.byref(fwd), ctypes.byref(bwd)),
            "asa_stable_workspace_bytes")
    ws = torch.empty(bwd.value, device=dev, dtype=torch.uint8)
    check_device_errors(dev)
    L.check(L.lib().asa_stable_backward(ctypes.byref(p), _ptr(Q), _ptr(K), _ptr(V), _ptr(s.top_val),
                                        _ptr(s.top_idx), _ptr(s.weights), _ptr(s.tau), _ptr(s.tau_coef),
                                        _ptr(dO), _ptr(dQ), _ptr(dK), _ptr(dV), _ptr(ws), bwd.value,
                                        _stream()),
            "asa_stable_backward")
    _poll_device_errors(dev)
    return dQ, dK, dV
