"""ctypes binding of the engine's C ABI (include/asa.h, libasa.so).

The library is the only compute path: if it is missing or fails to load, the
import fails loudly.  There is no CPU or eager-PyTorch fallback.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libasa.so")

ASA_OK, ASA_ERR_INVALID, ASA_ERR_UNSUPPORTED, ASA_ERR_WORKSPACE, ASA_ERR_CUDA, \
    ASA_ERR_DEVICE_TIMEOUT = range(6)
DTYPE_F32, DTYPE_BF16 = 0, 1
BACKEND = {"auto": 0, "simt": 1, "tc": 2}
BACKEND_NAME = {v: k for k, v in BACKEND.items()}
PRECISION = {"split": 0, "bf16": 1}
TAU_MODE = {"reference": 0, "exact": 1}
GRAD_MODE = {"reference": 0, "jacobian": 1}

#: the exported symbols include/asa.h declares
SYMBOLS = ("asa_params_default", "asa_workspace_bytes", "asa_resolve_backend", "asa_tau_mask",
           "asa_forward", "asa_backward", "asa_scrub", "asa_device_error", "asa_status_string",
           "asa_version", "asa_profile_begin", "asa_profile_end", "asa_profile_get",
           "asa_launch_count", "asa_last_cuda_error", "asa_tau_mask_noalloc",
           "asa_device_error_async", "asa_wait_probe", "asa_stable_workspace_bytes",
           "asa_stable_forward", "asa_stable_backward")
NOALLOC_SCRATCH_BYTES = 1 << 20


class Params(ctypes.Structure):
    """Mirror of struct asa_params (include/asa.h)."""
    _fields_ = [("B", ctypes.c_int), ("H", ctypes.c_int), ("NQ", ctypes.c_int),
                ("NK", ctypes.c_int), ("d", ctypes.c_int), ("block_m", ctypes.c_int),
                ("block_n", ctypes.c_int), ("k_keep", ctypes.c_int), ("alpha", ctypes.c_float),
                ("sm_scale", ctypes.c_float), ("causal", ctypes.c_int),
                ("in_dtype", ctypes.c_int), ("out_dtype", ctypes.c_int),
                ("backend", ctypes.c_int), ("precision", ctypes.c_int),
                ("timeout_spins", ctypes.c_longlong), ("ref_tile_load", ctypes.c_int),
                ("tau_mode", ctypes.c_int), ("grad_mode", ctypes.c_int),
                ("fused_forward", ctypes.c_int)]


class AsaError(RuntimeError):
    """A non-zero asa_status from the library.  Subclasses RuntimeError, the
    exception type the reference's TORCH_CHECKs raise."""

    def __init__(self, code, what):
        self.code = code
        extra = ""
        if code == ASA_ERR_CUDA:
            extra = f": {lib().asa_last_cuda_error().decode()}"
        super().__init__(f"{what}: {status_string(code)}{extra} (asa_status {code})")


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"splash_attention: {LIB_PATH} is missing; build it with "
                "`python adaptive-splash-attention_b200/build.py` (no fallback path exists)")
        L = ctypes.CDLL(LIB_PATH)
        vp, sz = ctypes.c_void_p, ctypes.c_size_t
        pp = ctypes.POINTER(Params)
        L.asa_params_default.argtypes = [pp]
        L.asa_params_default.restype = None
        L.asa_workspace_bytes.argtypes = [pp, ctypes.POINTER(sz), ctypes.POINTER(sz)]
        L.asa_resolve_backend.argtypes = [pp]
        L.asa_tau_mask.argtypes = [pp, vp, vp, vp, vp, vp, vp, vp, vp, vp, sz, vp]
        L.asa_forward.argtypes = [pp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, sz, vp]
        L.asa_backward.argtypes = [pp] + [vp] * 15 + [vp, sz, vp]
        L.asa_scrub.argtypes = [ctypes.c_int, vp, sz, vp, vp]
        L.asa_device_error.argtypes = [vp, ctypes.POINTER(ctypes.c_int)]
        L.asa_status_string.argtypes = [ctypes.c_int]
        L.asa_status_string.restype = ctypes.c_char_p
        L.asa_version.argtypes = []
        L.asa_profile_begin.argtypes = [ctypes.c_int]
        L.asa_profile_end.argtypes = []
        L.asa_profile_get.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_char_p),
                                      ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int)]
        L.asa_launch_count.argtypes = []
        L.asa_launch_count.restype = ctypes.c_longlong
        L.asa_tau_mask_noalloc.argtypes = [pp, vp, vp, vp, vp, vp, vp, vp, vp, vp]
        L.asa_device_error_async.argtypes = [vp, ctypes.POINTER(ctypes.c_int)]
        L.asa_wait_probe.argtypes = [ctypes.c_longlong, vp]
        L.asa_stable_workspace_bytes.argtypes = [pp, ctypes.POINTER(sz), ctypes.POINTER(sz)]
        L.asa_stable_forward.argtypes = [pp] + [vp] * 11 + [vp, sz, vp]
        L.asa_stable_backward.argtypes = [pp] + [vp] * 12 + [vp, sz, vp]
        L.asa_last_cuda_error.argtypes = []
        L.asa_last_cuda_error.restype = ctypes.c_char_p
        for name in SYMBOLS:
            getattr(L, name)
        _lib = L
    return _lib


def status_string(code):
    return lib().asa_status_string(int(code)).decode()


def check(code, what):
    if code != ASA_OK:
        raise AsaError(code, what)
