"""Build the reference's CUDA kernels (source/adasplashattention.cu, read in
place from the reference checkout) into oracle/_ref/<variant>/.

TEST INFRASTRUCTURE ONLY.  Runs in the development container, where the
reference checkout exists; the built .so files travel to the GPU box and are
loaded there by tests/golden/make_golden.py.  Flags: -O2
--expt-relaxed-constexpr, no fast-math (the reference ships no build flags;
torch's default has no fast-math).  Tile sizes and K_KEEP are the
reference's compile-time macros (adasplashattention.cu:8-19), so each
variant is a separate module.

    python oracle/build_ref.py [--ref-src DIR]
"""
import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")

# (name, BLOCK_M, BLOCK_N, K_KEEP)
VARIANTS = [
    ("m64n64k8", 64, 64, 8),
    ("m32n64k8", 32, 64, 8),
    ("m32n32k8", 32, 32, 8),
    ("m32n64k16", 32, 64, 16),
]


def build_variant(name, bm, bn, kk, ref_src):
    from torch.utils.cpp_extension import load
    bdir = os.path.join(OUT, name)
    os.makedirs(bdir, exist_ok=True)
    defs = [f"-DBLOCK_M={bm}", f"-DBLOCK_N={bn}", f"-DK_KEEP={kk}", f"-DREF_OPS_NS=asa_ref_{name}"]
    load(name=f"asa_ref_{name}", sources=[os.path.join(HERE, "ref_wrapper.cu")],
         extra_include_paths=[ref_src], build_directory=bdir, verbose=False,
         extra_cflags=["-O2"] + defs,
         extra_cuda_cflags=["-O2", "--expt-relaxed-constexpr",
                            "-gencode", "arch=compute_100a,code=sm_100a"] + defs,
         is_python_module=True)
    return os.path.join(bdir, f"asa_ref_{name}.so")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-src", default=os.environ.get("ASA_REF_SRC", "/root/reference/source"))
    ap.add_argument("--only", default=None)
    a = ap.parse_args()
    if not os.path.exists(os.path.join(a.ref_src, "adasplashattention.cu")):
        print("reference source not found; nothing built", file=sys.stderr)
        return 1
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    for name, bm, bn, kk in VARIANTS:
        if a.only and name != a.only:
            continue
        print(build_variant(name, bm, bn, kk, a.ref_src), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
