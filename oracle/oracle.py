"""numpy front-end over the C oracle (asa_oracle.c).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  Arrays are float32 /
int32, laid out [BH, N, d] and [BH, N] like the reference's tensors
(source/adasplashattention.cu:558-567).
"""
import ctypes
import os

import numpy as np

from . import build as _build


class _Cfg(ctypes.Structure):
    _fields_ = [("BH", ctypes.c_int), ("NQ", ctypes.c_int), ("NK", ctypes.c_int),
                ("d", ctypes.c_int), ("BM", ctypes.c_int), ("BN", ctypes.c_int),
                ("k_keep", ctypes.c_int), ("alpha", ctypes.c_float),
                ("sm_scale", ctypes.c_float), ("causal", ctypes.c_int),
                ("ref_tile_load", ctypes.c_int)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.LIB
        if not os.path.exists(path):
            path = _build.build()
        _lib = ctypes.CDLL(path)
        f32p = np.ctypeslib.ndpointer(np.float32, flags="C")
        i32p = np.ctypeslib.ndpointer(np.int32, flags="C")
        u8p = np.ctypeslib.ndpointer(np.uint8, flags="C")
        cfgp = ctypes.POINTER(_Cfg)
        _lib.asa_oracle_entmax_tau.argtypes = [f32p, ctypes.c_int, ctypes.c_float]
        _lib.asa_oracle_entmax_tau.restype = ctypes.c_float
        _lib.asa_oracle_tau_mask.argtypes = [cfgp, f32p, f32p, i32p, i32p, f32p, u8p,
                                             ctypes.c_void_p, ctypes.c_void_p]
        _lib.asa_oracle_csr.argtypes = [cfgp, u8p, i32p, i32p]
        _lib.asa_oracle_forward.argtypes = [cfgp, f32p, f32p, f32p, i32p, i32p, f32p, i32p, i32p,
                                            f32p, ctypes.c_void_p]
        _lib.asa_oracle_backward.argtypes = [cfgp, f32p, f32p, f32p, i32p, i32p, f32p, i32p, i32p,
                                             f32p, f32p, f32p, f32p]
        _lib.asa_oracle_stable_forward.argtypes = [cfgp, f32p, f32p, i32p, f32p, f32p, f32p, f32p]
    return _lib


class Config:
    """Shape and settings of one call.  The reference's compile-time
    BLOCK_M / BLOCK_N / K_KEEP (source/adasplashattention.cu:8-19) are runtime
    fields here."""

    def __init__(self, BH, NQ, NK, d, BM=128, BN=128, k_keep=8, alpha=1.5, sm_scale=None,
                 causal=True, ref_tile_load=True):
        self.BH, self.NQ, self.NK, self.d = int(BH), int(NQ), int(NK), int(d)
        self.BM, self.BN, self.k_keep = int(BM), int(BN), int(k_keep)
        self.alpha = float(alpha)
        self.sm_scale = float(sm_scale if sm_scale is not None else d ** -0.5)
        self.causal = bool(causal)
        # reproduce the reference's tile-load zeroing (asa_oracle.c row_of)
        self.ref_tile_load = bool(ref_tile_load)
        self.nQB = -(-self.NQ // self.BM)
        self.nKB = -(-self.NK // self.BN)

    def c(self):
        return _Cfg(self.BH, self.NQ, self.NK, self.d, self.BM, self.BN, self.k_keep,
                    self.alpha, self.sm_scale, int(self.causal), int(self.ref_tile_load))


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


def entmax_tau(s, alpha):
    """τ of one sorted-descending top-k list (reference entmax_threshold)."""
    s = _f32(s)
    return float(lib().asa_oracle_entmax_tau(s, s.size, alpha))


def tau_mask(cfg, Q, K, Qidx, Kidx, want_topk=False):
    Q, K = _f32(Q).reshape(cfg.BH, cfg.NQ, cfg.d), _f32(K).reshape(cfg.BH, cfg.NK, cfg.d)
    Qidx, Kidx = _i32(Qidx).reshape(cfg.BH, cfg.NQ), _i32(Kidx).reshape(cfg.BH, cfg.NK)
    tau = np.zeros((cfg.BH, cfg.NQ), np.float32)
    M = np.zeros((cfg.BH, cfg.nQB, cfg.nKB), np.uint8)
    topv = np.zeros((cfg.BH, cfg.NQ, cfg.k_keep), np.float32) if want_topk else None
    topi = np.zeros((cfg.BH, cfg.NQ, cfg.k_keep), np.int32) if want_topk else None
    c = cfg.c()
    lib().asa_oracle_tau_mask(ctypes.byref(c), Q, K, Qidx, Kidx, tau, M,
                              topv.ctypes.data if want_topk else None,
                              topi.ctypes.data if want_topk else None)
    if want_topk:
        return tau, M, topv, topi
    return tau, M


def csr(cfg, M):
    M = np.ascontiguousarray(M, dtype=np.uint8)
    ptr = np.zeros((cfg.BH, cfg.nQB + 1), np.int32)
    idx = np.zeros((cfg.BH, cfg.nQB * cfg.nKB), np.int32)
    c = cfg.c()
    lib().asa_oracle_csr(ctypes.byref(c), M, ptr, idx)
    return ptr, idx


def forward(cfg, Q, K, V, Qidx, Kidx, tau, ptr, idx, want_rownorm=False):
    Q, K, V = (_f32(x) for x in (Q, K, V))
    O = np.zeros((cfg.BH, cfg.NQ, cfg.d), np.float32)
    n = np.zeros((cfg.BH, cfg.NQ), np.float32) if want_rownorm else None
    c = cfg.c()
    lib().asa_oracle_forward(ctypes.byref(c), Q, K, V, _i32(Qidx), _i32(Kidx), _f32(tau),
                             _i32(ptr), _i32(idx), O, n.ctypes.data if want_rownorm else None)
    return (O, n) if want_rownorm else O


def host_scrub(x):
    """The reference launchers' post-kernel scrub (adasplashattention.cu:599-606,
    684-697): NaN -> 0, then, if any Inf remains, clamp the WHOLE tensor to
    [-100, 100]."""
    x = np.where(np.isnan(x), np.float32(0), x)
    if np.isinf(x).any():
        x = np.clip(x, -100.0, 100.0).astype(np.float32)
    return x


def backward(cfg, Q, K, V, Qidx, Kidx, tau, ptr, idx, dO):
    Q, K, V, dO = (_f32(x) for x in (Q, K, V, dO))
    dQ = np.zeros((cfg.BH, cfg.NQ, cfg.d), np.float32)
    dK = np.zeros((cfg.BH, cfg.NK, cfg.d), np.float32)
    dV = np.zeros((cfg.BH, cfg.NK, cfg.d), np.float32)
    c = cfg.c()
    lib().asa_oracle_backward(ctypes.byref(c), Q, K, V, _i32(Qidx), _i32(Kidx), _f32(tau),
                              _i32(ptr), _i32(idx), dO, dQ, dK, dV)
    return host_scrub(dQ), host_scrub(dK), host_scrub(dV)


def run_all(cfg, Q, K, V, Qidx, Kidx, dO=None):
    """τ/mask → CSR → forward (→ backward): the reference's forward_splash /
    backward_splash sequences (adasplashattention.cu:537-609, 611-700)."""
    tau, M = tau_mask(cfg, Q, K, Qidx, Kidx)
    ptr, idx = csr(cfg, M)
    O, n = forward(cfg, Q, K, V, Qidx, Kidx, tau, ptr, idx, want_rownorm=True)
    out = dict(tau=tau, M=M, ptr=ptr, idx=idx, O=host_scrub(O), rownorm=n)
    if dO is not None:
        out["dQ"], out["dK"], out["dV"] = backward(cfg, Q, K, V, Qidx, Kidx, tau, ptr, idx, dO)
    return out


def stable_forward(cfg, Q, K, V, Qidx, Kidx):
    """The notebook's top-k-only ("stable") operator: the top-k lists of
    tau_mask (without the reference's tile-load zeroing, as the notebook
    kernel reads K directly), then its bisection τ, weights and output."""
    import copy
    c0 = copy.copy(cfg)
    c0.ref_tile_load = False
    _, _, topv, topi = tau_mask(c0, Q, K, Qidx, Kidx, want_topk=True)
    rows = cfg.BH * cfg.NQ
    O = np.zeros((cfg.BH, cfg.NQ, cfg.d), np.float32)
    tau = np.zeros(rows, np.float32)
    coef = np.zeros(rows, np.float32)
    w = np.zeros((rows, cfg.k_keep), np.float32)
    c = c0.c()
    lib().asa_oracle_stable_forward(ctypes.byref(c), _f32(V), np.ascontiguousarray(topv, np.float32),
                                    np.ascontiguousarray(topi, np.int32), O, tau, w, coef)
    return dict(O=O, tau=tau.reshape(cfg.BH, cfg.NQ), weights=w.reshape(cfg.BH, cfg.NQ, -1),
                tau_coef=coef.reshape(cfg.BH, cfg.NQ), topv=topv, topi=topi)
