"""Build the engine's C-ABI library (libasa.so) for sm_100a with nvcc.

    python adaptive-splash-attention_b200/build.py [--force]

Objects go to adaptive-splash-attention_b200/_build/; the library lands in
adaptive-splash-attention_b200/splash_attention/libasa.so, next to the
Python package that loads it, and the PyTorch operator library over it in
splash_attention/_torch_ops.so.
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
SOURCES = ["asa_capi.cu", "asa_simt.cu", "asa_compact.cu", "asa_stable.cu"]
# asa_tc.cu is compiled as five objects (τ/mask, forward, dQ, dK/dV, fused
# forward) so the template instantiations build in parallel.
TC_PARTS = [("asa_tc.cu", part) for part in (1, 2, 3, 4, 5)]


def _deps():
    return [os.path.join(CSRC, f) for f in os.listdir(CSRC)
            if f.endswith((".cu", ".cuh", ".h"))] + [
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


TORCH_OPS = os.path.join(HERE, "splash_attention", "_torch_ops.so")


def build_torch_ops(force: bool = False) -> str:
    """The TORCH_LIBRARY operators (csrc/torch_ops.cpp): host C++ against
    PyTorch's headers, linked to libasa.so (found next to it at run time)."""
    import torch
    import torch.utils.cpp_extension as ce
    src = os.path.join(CSRC, "torch_ops.cpp")
    deps = [src, os.path.join(HERE, "..", "include", "asa.h"), LIB]
    if (not force and os.path.exists(TORCH_OPS)
            and os.path.getmtime(TORCH_OPS) >= max(os.path.getmtime(p) for p in deps)):
        return TORCH_OPS
    cuda_home = os.path.dirname(os.path.dirname(NVCC))
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           src, "-o", TORCH_OPS + ".tmp", "-I", os.path.join(cuda_home, "include")]
    for p in ce.include_paths():
        cmd += ["-isystem", p]
    for p in ce.library_paths():
        cmd += ["-L", p, f"-Wl,-rpath,{p}"]
    cmd += ["-L", os.path.dirname(LIB), "-l:libasa.so", "-Wl,-rpath,$ORIGIN",
            "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"g++ failed for torch_ops.cpp:\n{r.stdout}\n{r.stderr}")
    os.replace(TORCH_OPS + ".tmp", TORCH_OPS)
    return TORCH_OPS


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
    print(build_torch_ops(force="--force" in sys.argv))
