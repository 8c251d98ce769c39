"""The C-ABI library loads and exports what include/asa.h declares; argument
checks run without a GPU."""
import ctypes
import os
import re

import pytest

from splash_attention import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    text = open(os.path.join(ROOT, "include", "asa.h")).read()
    return set(re.findall(r"^\s*(?:int|void|const char\*|long long)\s+(asa_\w+)\s*\(", text, re.M))


def test_exports_every_declared_symbol():
    lib = L.lib()
    declared = header_functions()
    assert declared == set(L.SYMBOLS)
    for name in declared:
        assert hasattr(lib, name), name


def params(**kw):
    p = L.Params()
    L.lib().asa_params_default(ctypes.byref(p))
    p.B, p.H, p.NQ, p.NK, p.d, p.sm_scale = 2, 4, 1024, 1024, 128, 128 ** -0.5
    for k, v in kw.items():
        setattr(p, k, v)
    return p


def ws(p):
    f, b = ctypes.c_size_t(), ctypes.c_size_t()
    rc = L.lib().asa_workspace_bytes(ctypes.byref(p), ctypes.byref(f), ctypes.byref(b))
    return rc, f.value, b.value


def test_defaults():
    p = params()
    assert (p.block_m, p.block_n, p.k_keep, p.causal) == (128, 128, 8, 1)
    assert abs(p.alpha - 1.5) < 1e-7
    rc, f, b = ws(p)
    assert rc == 0 and f % 16 == 0 and b % 16 == 0 and b > 0


@pytest.mark.parametrize("field,value,code", [
    ("d", 0, L.ASA_ERR_INVALID), ("d", 129, L.ASA_ERR_UNSUPPORTED),
    ("k_keep", 0, L.ASA_ERR_INVALID), ("k_keep", 33, L.ASA_ERR_UNSUPPORTED),
    ("block_m", 0, L.ASA_ERR_INVALID), ("B", 0, L.ASA_ERR_INVALID),
    ("in_dtype", 7, L.ASA_ERR_INVALID), ("backend", 9, L.ASA_ERR_INVALID),
    ("alpha", float("nan"), L.ASA_ERR_INVALID), ("NQ", -1, L.ASA_ERR_INVALID),
])
def test_rejects_bad_params(field, value, code):
    assert ws(params(**{field: value}))[0] == code


def test_k_keep_cannot_exceed_block_n():
    # reference static_assert(K_KEEP <= BLOCK_N) (:32)
    assert ws(params(block_n=4, k_keep=8))[0] == L.ASA_ERR_INVALID


def test_backend_resolution():
    lib = L.lib()
    simt = params(in_dtype=L.DTYPE_F32)
    assert lib.asa_resolve_backend(ctypes.byref(params(backend=1))) == 1
    assert lib.asa_resolve_backend(ctypes.byref(simt)) in (1,)
    assert lib.asa_resolve_backend(ctypes.byref(params(d=0))) == -L.ASA_ERR_INVALID


def test_status_strings():
    assert L.status_string(0) == "ok"
    assert "workspace" in L.status_string(L.ASA_ERR_WORKSPACE)
