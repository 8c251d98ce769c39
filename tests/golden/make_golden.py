"""Generate tests/golden/*.npz by running the reference's own CUDA kernels.

Run on a GPU box after `python oracle/build_ref.py` built the reference
modules into oracle/_ref/ (the built .so files travel with the repository
snapshot; the reference checkout itself is not read here):

    python tests/golden/make_golden.py [--out DIR]

Per case it stores τ, M, Qi_ptr, Qi_idx (via the wrapper's mask_tau op, which
launches the reference's build_mask_kernel / build_lookup_kernel), O from the
reference pybind ``forward`` and dQ, dK, dV from its ``backward``.
"""
import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
from cases import CASES, spec, make_inputs, checksum  # noqa: E402

_mods = {}


def ref_module(variant):
    if variant not in _mods:
        path = os.path.join(ROOT, "oracle", "_ref", variant, f"asa_ref_{variant}.so")
        sp = importlib.util.spec_from_file_location(f"asa_ref_{variant}", path)
        m = importlib.util.module_from_spec(sp)
        sp.loader.exec_module(m)
        _mods[variant] = m
    return _mods[variant]


def run_case(name):
    s = spec(name)
    m = ref_module(s["variant"])
    ops = getattr(torch.ops, f"asa_ref_{s['variant']}")
    Q, K, V, dO, Qi, Ki = make_inputs(name)
    dev = "cuda"
    Qd, Kd, Vd, dOd, Qid, Kid = (x.to(dev).contiguous() for x in (Q, K, V, dO, Qi, Ki))
    tau, M, ptr, idx = ops.mask_tau(Qd, Kd, Qid, Kid, s["sm_scale"], s["alpha"])
    O = m.forward(Qd, Kd, Vd, Qid, Kid, s["sm_scale"], s["alpha"])
    dQ, dK, dV = m.backward(Qd, Kd, Vd, Qid, Kid, s["sm_scale"], s["alpha"], dOd)
    torch.cuda.synchronize()
    out = dict(tau=tau, M=M, ptr=ptr, idx=idx, O=O, dQ=dQ, dK=dK, dV=dV)
    out = {k: v.cpu().numpy() for k, v in out.items()}
    out["M"] = out["M"].astype(np.uint8)
    out["input_checksum"] = np.float64(checksum(Q, K, V, dO))
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=HERE)
    a = ap.parse_args()
    os.makedirs(a.out, exist_ok=True)
    for name in CASES:
        out = run_case(name)
        np.savez_compressed(os.path.join(a.out, f"{name}.npz"), **out)
        print(name, {k: getattr(v, "shape", v) for k, v in out.items()}, flush=True)


if __name__ == "__main__":
    main()
