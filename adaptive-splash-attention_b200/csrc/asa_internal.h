// asa_internal.h -- launch-side declarations shared by the C-ABI translation
// unit and the kernel translation units.  Not part of the public ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include "asa_device.cuh"
#include "../../include/asa.h"

namespace asa {

// Everything a kernel needs to know about one call, resolved on the host.
struct Shape {
    int BH, NQ, NK, d;
    int BM, BN, k;
    int causal;
    int nQB, nKB;
    float alpha;     // clamped to [1.05, 3] (reference :547)
    float am1;       // α - 1
    float inv_am1b;  // 1/(α-1) as the backward forms it (:499)
    float scale;
    PowSpec pinv;    // exponent 1/(α-1)          (:312)
    PowSpec pe2;     // exponent (2-α)/(α-1)      (:495)
    long long spins; // bound on device-side waits
    int in_dtype, out_dtype;
    int ref_load;    // reproduce the reference's tile-load zeroing (causal only)
    int split;       // tcgen05 path: P and dS enter the MMAs as bf16 hi+lo pairs
    int exact_tau;   // asa_tau_mode ASA_TAU_EXACT
    int jacobian;    // asa_grad_mode ASA_GRAD_JACOBIAN
};

// Passes of the exact-τ solve: one for the row maximum, then Newton steps
// (bisection-safeguarded) on Σ u_+^{1/(α-1)} = 1 from the left end of the
// bracket [(α-1)s_max - 1, (α-1)s_max].
constexpr int kExactPasses = 10;

// Whether element `t` of key row `kn` survives the reference's tile staging
// for consumers in query block `qb`: the reference thread that stages it
// serves query qb*BM + ((kn % BN)*d + t) % BM and zeroes it when that query
// cannot see the key (source/adasplashattention.cu:176-183, :285-294,
// :398-406, :442-450).  A staging query >= NQ has no reference thread (it
// exits first, :156-158); the element is then kept.
__device__ __forceinline__ bool ref_keep(const Shape& s, const int32_t* __restrict__ Qidx_bh,
                                         int qb, int kn, int t, int kpos) {
    const int lq = qb * s.BM + (int)(((long long)(kn % s.BN) * s.d + t) % s.BM);
    return lq >= s.NQ || kpos <= __ldg(Qidx_bh + lq);
}

// Count of kernels this library has launched (for the bench's launch
// count); every launch site calls note_launch().
void note_launch(int n = 1);

// ---- SIMT kernels (asa_simt.cu) -------------------------------------------
// topv / topi (optional): each row's top-k scores and keys in order.
cudaError_t simt_tau_mask(const Shape& s, const void* Q, const void* K, const int32_t* Qidx,
                          const int32_t* Kidx, float* tau, uint8_t* M, cudaStream_t st,
                          float* topv = nullptr, int32_t* topi = nullptr);
cudaError_t simt_forward(const Shape& s, const void* Q, const void* K, const void* V,
                         const int32_t* Qidx, const int32_t* Kidx, const float* tau,
                         const int32_t* ptr, const int32_t* idx, void* O, float* O32,
                         float* rownorm, cudaStream_t st);
cudaError_t simt_rowstats(const Shape& s, const void* Q, const void* K, const void* V,
                          const int32_t* Qidx, const int32_t* Kidx, const float* tau,
                          const int32_t* ptr, const int32_t* idx, const void* dO,
                          float* invN, float* accdO, cudaStream_t st);
cudaError_t simt_dq(const Shape& s, const void* Q, const void* K, const void* V,
                    const int32_t* Qidx, const int32_t* Kidx, const float* tau,
                    const int32_t* ptr, const int32_t* idx, const void* dO,
                    const float* invN, const float* accdO, void* dQ, cudaStream_t st);
cudaError_t simt_dkdv(const Shape& s, const void* Q, const void* K, const void* V,
                      const int32_t* Qidx, const int32_t* Kidx, const float* tau,
                      const int32_t* cptr, const int32_t* cidx, const void* dO,
                      const float* invN, const float* accdO, void* dK, void* dV,
                      cudaStream_t st);

cudaError_t simt_exact_tau(const Shape& s, const void* Q, const void* K, const int32_t* Qidx,
                           const int32_t* Kidx, float* tau, uint8_t* M, cudaStream_t st);
cudaError_t simt_jacobian_stats(const Shape& s, const void* Q, const void* K, const void* V,
                                const int32_t* Qidx, const int32_t* Kidx, const float* tau,
                                const int32_t* ptr, const int32_t* idx, const void* dO,
                                float* invN, float* accdO, cudaStream_t st);

// ---- top-k-only ("stable") operator (asa_stable.cu) ---------------------------
// From each row's top-k scores and keys (in order): τ by the five-step
// bisection, the normalised weights, O = Σ_j w_j V[key_j]; and its gradient.
cudaError_t stable_forward(const Shape& s, float alpha, const void* V, const float* topv,
                           const int32_t* topi, void* O, float* tau, float* weights,
                           float* tau_coef, cudaStream_t st);
cudaError_t stable_backward(const Shape& s, float alpha, const void* Q, const void* K,
                            const void* V, const void* dO, const float* topv,
                            const int32_t* topi, const float* weights, const float* tau,
                            const float* tau_coef, void* dQ, float* dK32, float* dV32,
                            void* dK, void* dV, cudaStream_t st);

// ---- tile lists (asa_compact.cu) --------------------------------------------
// CSR of M in the reference's format (build_lookup_kernel :219-242), and the
// transposed list (per key block, the query blocks that use it) the backward
// walks.  Either output pair may be null.
cudaError_t build_lists(const Shape& s, const uint8_t* M, int32_t* csr_ptr, int32_t* csr_idx,
                        int32_t* csc_ptr, int32_t* csc_idx, cudaStream_t st);
// Device-side version of the reference host scrub (:599-606).
cudaError_t scrub(int dtype, void* x, size_t n, int* flag, cudaStream_t st);

}  // namespace asa
