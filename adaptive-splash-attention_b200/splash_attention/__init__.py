"""splash_attention -- B200 α-entmax block-sparse attention (AdaSplash path).

Drop-in surface of mvideet/Adaptive-Splash-Attention:

* ``AdaptiveSplashAttention(head_dim, alpha, k_keep, adaptive_threshold,
  sm_scale)`` called as ``attention(Q, K, V, Q_idx, K_idx)`` with autograd
  backward -- the module the reference's README describes
  (README.md:100-124; it ships no implementation of it);
* module-level ``forward(Q, K, V, Q_idx, K_idx, sm_scale, alpha)`` and
  ``backward(Q, K, V, Q_idx, K_idx, sm_scale, alpha, dOut)`` with the
  signatures of the reference's pybind module
  (source/adasplashattention.cu:702-705), using the reference's default
  build settings (BLOCK_M=32, BLOCK_N=64, K_KEEP=8, :8-19) and its host-side
  NaN/Inf scrub.

Every computation runs in hand-written CUDA kernels for sm_100a behind the C
ABI of include/asa.h (libasa.so).  There is no CPU fallback.
"""
import os

import torch

from . import _lib
from .ops import Settings, forward_saved, backward_saved, tau_mask, scrub_, device_error, \
    resolved_backend, make_params, _index, _check_inputs, stable_forward_saved, stable_backward_saved
from .streamed import forward_backward_host

_lib.lib()  # fail at import time if the native library is missing

_TORCH_OPS = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_torch_ops.so")
if not os.path.exists(_TORCH_OPS):
    raise ImportError(f"splash_attention: {_TORCH_OPS} is missing; build it with "
                      "`python adaptive-splash-attention_b200/build.py` (no fallback path exists)")
torch.ops.load_library(_TORCH_OPS)
_ops = torch.ops.splash_attention

__all__ = ["AdaptiveSplashAttention", "splash_attention", "forward", "backward", "tau_mask",
           "Settings", "device_error", "forward_backward_host", "stable_attention", "stable_forward",
           "stable_backward"]

# Reference compile-time defaults (adasplashattention.cu:8-19).
REF_BLOCK_M, REF_BLOCK_N, REF_K_KEEP = 32, 64, 8


def _op_config(Q, st: Settings):
    """The scalar arguments of splash_attention::forward / ::backward."""
    out_dt = st.out_dtype if st.out_dtype is not None else Q.dtype
    if out_dt not in (torch.float32, torch.bfloat16):
        raise TypeError(f"splash_attention: unsupported out_dtype {out_dt}")
    sm_scale = st.sm_scale if st.sm_scale is not None else Q.shape[-1] ** -0.5
    if st.tau_mode not in _lib.TAU_MODE or st.grad_mode not in _lib.GRAD_MODE:
        raise ValueError(f"splash_attention: tau_mode in {tuple(_lib.TAU_MODE)}, "
                         f"grad_mode in {tuple(_lib.GRAD_MODE)}")
    return (float(st.alpha), float(sm_scale), int(st.k_keep), int(st.block_m), int(st.block_n),
            bool(st.causal), _lib.BACKEND[st.backend], _lib.PRECISION[st.precision],
            out_dt == torch.float32, bool(st.ref_tile_load), _lib.TAU_MODE[st.tau_mode],
            _lib.GRAD_MODE[st.grad_mode])


def _setup_context(ctx, inputs, output):
    Q, K, V, Qi, Ki = inputs[:5]
    O, O32, tau, M, ptr, idx, rown = output
    ctx.mark_non_differentiable(O32, tau, M, ptr, idx, rown)
    ctx.save_for_backward(Q, K, V, Qi, Ki, O32 if O32.numel() else O, tau, M, ptr, idx, rown)
    ctx.cfg = tuple(inputs[5:-2])      # everything but fused_forward and need_o32


def _backward(ctx, dO, *_unused):
    Q, K, V, Qi, Ki, O32, tau, M, ptr, idx, rown = ctx.saved_tensors
    if dO is None:
        return (None,) * 19
    dQ, dK, dV = _ops.backward(Q, K, V, Qi, Ki, O32, tau, M, ptr, idx, rown, dO, *ctx.cfg)
    return (dQ.to(Q.dtype), dK.to(K.dtype), dV.to(V.dtype)) + (None,) * 16


torch.library.register_autograd("splash_attention::forward", _backward,
                                setup_context=_setup_context)


def splash_attention(Q, K, V, Q_idx=None, K_idx=None, *, alpha=1.5, sm_scale=None, k_keep=8,
                     block_m=128, block_n=128, causal=True, backend="auto", precision="split",
                     out_dtype=None, ref_tile_load=True, tau_mode="reference", grad_mode="reference",
                     fused_forward=True):
    """α-entmax block-sparse attention with autograd.  Q, K, V: [B, H, N, d]
    float32 or bfloat16 on CUDA; Q_idx / K_idx: positions [B*H, N] (any
    integer dtype; [N] broadcasts).  Key k is visible to query q iff
    K_idx[k] <= Q_idx[q] (causal=False: every key).

    Runs the registered operator splash_attention::forward (C++ over the C
    ABI; traceable through its Meta kernel), whose autograd formula calls
    splash_attention::backward.

    ref_tile_load=True reproduces the reference kernels' tile staging, in
    which a visible key's K/V elements are zeroed when the reference thread
    that loads them serves a query that cannot see the key; False reads every
    visible key in full.

    tau_mode="exact" replaces the reference's top-k threshold by the exact
    α-entmax threshold over every visible key (and the mask by every tile
    holding a positive weight); grad_mode="jacobian" replaces the fixed-τ
    gradient by the α-entmax Jacobian.  Both together give exact α-entmax
    attention and its exact gradient.

    fused_forward=True runs the tcgen05 forward (bf16 output, k_keep <= 8,
    reference τ) as one kernel per query block -- τ / mask and the forward
    together; False runs them as separate launches.  The outputs agree
    either way."""
    st = Settings(alpha=alpha, sm_scale=sm_scale, k_keep=k_keep, block_m=block_m,
                  block_n=block_n, causal=causal, backend=backend, precision=precision,
                  out_dtype=out_dtype, ref_tile_load=ref_tile_load, tau_mode=tau_mode,
                  grad_mode=grad_mode)
    if Q.device.type != "meta":
        _check_inputs(Q, K, V)
    BH = Q.shape[0] * Q.shape[1]
    qi = _index(Q_idx, BH, Q.shape[2], Q.device, "Q_idx") if causal else None
    ki = _index(K_idx, BH, K.shape[2], Q.device, "K_idx") if causal else None
    need_o32 = torch.is_grad_enabled() and any(t.requires_grad for t in (Q, K, V))
    return _ops.forward(Q, K, V, qi, ki, *_op_config(Q, st), bool(fused_forward), need_o32)[0]


class AdaptiveSplashAttention(torch.nn.Module):
    """The README's module (README.md:104-124).

    ``adaptive_threshold``: the reference has no implementation of it (the τ
    solve always runs).  True is accepted and means exactly that; False is
    rejected because no fixed-threshold semantics exist to reproduce.
    The module holds no parameters."""

    def __init__(self, head_dim, alpha=1.5, k_keep=8, adaptive_threshold=True, sm_scale=None,
                 block_m=128, block_n=128, causal=True, backend="auto", precision="split",
                 out_dtype=None, ref_tile_load=True, tau_mode="reference", grad_mode="reference"):
        super().__init__()
        if not adaptive_threshold:
            raise ValueError("AdaptiveSplashAttention: adaptive_threshold=False has no "
                             "reference semantics; only the per-query τ solve exists")
        if not 1 <= head_dim <= 128:
            raise ValueError("AdaptiveSplashAttention: head_dim must be in [1, 128]")
        self.head_dim = head_dim
        self.alpha = alpha
        self.k_keep = k_keep
        self.adaptive_threshold = adaptive_threshold
        self.sm_scale = sm_scale if sm_scale is not None else head_dim ** -0.5
        self.block_m, self.block_n = block_m, block_n
        self.causal = causal
        self.backend, self.precision, self.out_dtype = backend, precision, out_dtype
        self.ref_tile_load = ref_tile_load
        self.tau_mode, self.grad_mode = tau_mode, grad_mode

    def forward(self, Q, K, V, Q_idx=None, K_idx=None):
        if Q.shape[-1] != self.head_dim:
            raise ValueError(f"expected head_dim {self.head_dim}, got {Q.shape[-1]}")
        return splash_attention(Q, K, V, Q_idx, K_idx, alpha=self.alpha, sm_scale=self.sm_scale,
                                k_keep=self.k_keep, block_m=self.block_m,
                                block_n=self.block_n, causal=self.causal, backend=self.backend,
                                precision=self.precision, out_dtype=self.out_dtype,
                                ref_tile_load=self.ref_tile_load, tau_mode=self.tau_mode,
                                grad_mode=self.grad_mode)

    def extra_repr(self):
        return (f"head_dim={self.head_dim}, alpha={self.alpha}, k_keep={self.k_keep}, "
                f"sm_scale={self.sm_scale}, block=({self.block_m},{self.block_n}), "
                f"causal={self.causal}, backend={self.backend}, precision={self.precision}, "
                f"tau_mode={self.tau_mode}, grad_mode={self.grad_mode}")


def _ref_settings(sm_scale, alpha):
    return Settings(alpha=alpha, sm_scale=sm_scale, k_keep=REF_K_KEEP, block_m=REF_BLOCK_M,
                    block_n=REF_BLOCK_N, causal=True)


def forward(Q, K, V, Q_idx, K_idx, sm_scale, alpha):
    """Reference pybind ``forward`` (adasplashattention.cu:537-609, :703):
    returns O in Q's dtype, scrubbed as the reference's host code does."""
    O, _ = forward_saved(Q, K, V, Q_idx, K_idx, _ref_settings(sm_scale, alpha), need_o32=False)
    return scrub_(O)


def backward(Q, K, V, Q_idx, K_idx, sm_scale, alpha, dOut):
    """Reference pybind ``backward`` (adasplashattention.cu:611-700, :704):
    recomputes τ, the mask and the tile lists from scratch, returns
    [dQ, dK, dV] scrubbed like the reference's host code."""
    st = _ref_settings(sm_scale, alpha)
    _, saved = forward_saved(Q, K, V, Q_idx, K_idx, st, need_o32=True)
    grads = backward_saved(Q, K, V, dOut, saved)
    return [scrub_(g) for g in grads]


# ---- the notebook's top-k-only ("stable") operator -----------------------------
class _StableFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Q, K, V, Q_idx, K_idx, st):
        O, saved = stable_forward_saved(Q, K, V, Q_idx, K_idx, st)
        ctx.saved = saved
        ctx.save_for_backward(Q, K, V)
        return O

    @staticmethod
    def backward(ctx, dO):
        Q, K, V = ctx.saved_tensors
        dQ, dK, dV = stable_backward_saved(Q, K, V, dO, ctx.saved)
        return dQ.to(Q.dtype), dK.to(K.dtype), dV.to(V.dtype), None, None, None


def stable_attention(Q, K, V, Q_idx=None, K_idx=None, *, alpha=1.5, sm_scale=None, k_keep=8,
                     causal=True, backend="auto", out_dtype=None):
    """The reference notebook's top-k-only α-entmax attention
    (AdaSplashNotebook.ipynb, stable_splash_kernel): each query attends to
    its k_keep highest-scoring visible keys with bisection-τ α-entmax
    weights, O = Σ_j w_j V[key_j].  Autograd gives the operator's gradient
    (the notebook's backward returns zeros).  Q, K, V: [B, H, N, d] float32
    or bfloat16 on CUDA."""
    st = Settings(alpha=alpha, sm_scale=sm_scale, k_keep=k_keep, causal=causal, backend=backend,
                  out_dtype=out_dtype, ref_tile_load=False)
    return _StableFn.apply(Q, K, V, Q_idx, K_idx, st)


def stable_forward(Q, K, V, Q_idx, K_idx, sm_scale, alpha):
    """The notebook's stable module ``forward(Q, K, V, Q_idx, K_idx,
    sm_scale, alpha)`` (K_KEEP = 8): returns O in Q's dtype."""
    O, _ = stable_forward_saved(Q, K, V, Q_idx, K_idx,
                                Settings(alpha=alpha, sm_scale=sm_scale, k_keep=REF_K_KEEP,
                                         ref_tile_load=False))
    return O


def stable_backward(Q, K, V, Q_idx, K_idx, sm_scale, alpha, dOut):
    """The notebook's stable module ``backward(...)`` signature with the
    operator's gradient: returns [dQ, dK, dV]."""
    st = Settings(alpha=alpha, sm_scale=sm_scale, k_keep=REF_K_KEEP, ref_tile_load=False)
    _, saved = stable_forward_saved(Q, K, V, Q_idx, K_idx, st)
    return list(stable_backward_saved(Q, K, V, dOut, saved))
