"""Build the engine's C-ABI library (libasa.so) for sm_100a with nvcc.

    python adaptive-splash-attention_b200/build.py [--force]

Objects go to adaptive-splash-attention_b200/_build/; the library lands in
adaptive-splash-attention_b200/splash_attention/libasa.so, next to the
Python package that loads it.
"""
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "splash_attention", "libasa.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off", "--expt-relaxed-constexpr",
         "-Xptxas", "-v" if os.environ.get("ASA_PTXAS_V") else "-O3"]
SOURCES = ["asa_capi.cu", "asa_simt.cu", "asa_compact.cu"]
# asa_tc.cu is compiled as four objects (τ/mask, forward, dQ, dK/dV) so the
# template instantiations build in parallel.
TC_PARTS = [("asa_tc.cu", part) for part in (1, 2, 3, 4)]


def _deps():
    return [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [
        os.path.join(HERE, "..", "include", "asa.h")]


def _compile(item):
    src, part = item if isinstance(item, tuple) else (item, None)
    tag = f".part{part}" if part else ""
    obj = os.path.join(BUILD, os.path.basename(src) + tag + ".o")
    newest = max(os.path.getmtime(p) for p in _deps())
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest:
        return obj
    defs = [f"-DASA_TC_PART={part}"] if part else []
    cmd = [NVCC] + FLAGS + defs + ["-c", os.path.join(CSRC, src), "-o", obj + ".tmp"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if os.environ.get("ASA_PTXAS_V"):
        sys.stderr.write(r.stderr)
    os.replace(obj + ".tmp", obj)
    return obj


def build(force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    if force:
        for f in os.listdir(BUILD):
            os.remove(os.path.join(BUILD, f))
    items = SOURCES + TC_PARTS
    with cf.ThreadPoolExecutor(len(items)) as ex:
        objs = list(ex.map(_compile, items))
    if (not force and os.path.exists(LIB)
            and os.path.getmtime(LIB) >= max(os.path.getmtime(o) for o in objs)):
        return LIB
    cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB + ".tmp"] + objs
    subprocess.check_call(cmd)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
