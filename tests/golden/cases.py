"""Golden-vector cases: seeded inputs and the reference build each one runs on.

Each case names the reference module variant (compile-time BLOCK_M, BLOCK_N,
K_KEEP of source/adasplashattention.cu:8-19) built by oracle/build_ref.py.
Inputs are regenerated from the seed with torch's CPU generator (order Q, K,
V, dO; fp32 N(0, sigma²)), so the fixtures store outputs plus an input
checksum.
"""
import numpy as np
import torch

INT32_MAX = 2 ** 31 - 1

# name: (variant, BM, BN, KK, B, H, NQ, NK, d, alpha, sm_scale, causal, sigma, seed, bf16_round, qoff)
CASES = {
    "c1_m64n64": ("m64n64k8", 64, 64, 8, 1, 2, 256, 256, 64, 1.5, 0.125, True, 1.0, 0, False, 0),
    "c2s_m32n64": ("m32n64k8", 32, 64, 8, 1, 2, 512, 512, 64, 1.5, 0.125, True, 1.0, 1, False, 0),
    "d128_m32n32": ("m32n32k8", 32, 32, 8, 1, 2, 256, 256, 128, 1.5, 128 ** -0.5, True, 1.0, 2, False, 0),
    "bf16r_d128": ("m32n32k8", 32, 32, 8, 1, 2, 256, 256, 128, 1.5, 128 ** -0.5, True, 1.0, 3, True, 0),
    "alpha2": ("m32n64k8", 32, 64, 8, 1, 2, 256, 256, 64, 2.0, 0.125, True, 1.0, 4, False, 0),
    "alpha125": ("m32n64k8", 32, 64, 8, 1, 2, 256, 256, 64, 1.25, 0.125, True, 1.0, 5, False, 0),
    "alpha13": ("m32n64k8", 32, 64, 8, 1, 2, 256, 256, 64, 1.3, 0.125, True, 1.0, 6, False, 0),
    "noncausal_k16": ("m32n64k16", 32, 64, 16, 1, 2, 256, 256, 64, 1.5, 0.125, False, 2.0, 7, False, 0),
    "ragged": ("m32n64k8", 32, 64, 8, 1, 2, 200, 300, 64, 1.5, 0.125, True, 1.0, 8, False, 100),
    "saturated": ("m32n64k8", 32, 64, 8, 1, 1, 256, 256, 64, 1.5, 0.125, True, 3.0, 9, False, 0),
}


def spec(name):
    v, BM, BN, KK, B, H, NQ, NK, d, alpha, sm, causal, sigma, seed, bfr, qoff = CASES[name]
    return dict(variant=v, BM=BM, BN=BN, k_keep=KK, B=B, H=H, NQ=NQ, NK=NK, d=d, alpha=alpha,
                sm_scale=sm, causal=causal, sigma=sigma, seed=seed, bf16_round=bfr, qoff=qoff)


def make_inputs(name):
    """Q, K, V, dO as fp32 [B,H,N,d] CPU tensors and int32 [B*H, N] indices.
    Non-causal cases use Q_idx = INT32_MAX, the reference's only way to
    express it (every K_idx <= Q_idx)."""
    s = spec(name)
    g = torch.Generator().manual_seed(s["seed"])
    B, H, NQ, NK, d = s["B"], s["H"], s["NQ"], s["NK"], s["d"]
    Q = torch.randn(B, H, NQ, d, generator=g) * s["sigma"]
    K = torch.randn(B, H, NK, d, generator=g) * s["sigma"]
    V = torch.randn(B, H, NK, d, generator=g)
    dO = torch.randn(B, H, NQ, d, generator=g)
    if s["bf16_round"]:
        Q, K, V, dO = (x.bfloat16().float() for x in (Q, K, V, dO))
    BH = B * H
    if s["causal"]:
        Qi = (torch.arange(NQ, dtype=torch.int32) + s["qoff"]).expand(BH, NQ).contiguous()
    else:
        Qi = torch.full((BH, NQ), INT32_MAX, dtype=torch.int32)
    Ki = torch.arange(NK, dtype=torch.int32).expand(BH, NK).contiguous()
    return Q, K, V, dO, Qi, Ki


def checksum(*ts):
    return float(sum(float(t.double().abs().sum()) for t in ts))
