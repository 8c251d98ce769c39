// asa_simt.cu -- CUDA-core kernels of the engine.
//
// These kernels compute every score as the reference does: one fp32 FMA
// chain per (query, key) with the feature index ascending (reference
// source/adasplashattention.cu:190-193), so their scores, top-k picks, τ and
// block mask are bit-identical to the reference arithmetic for fp32 inputs.
// They serve fp32 inputs, any head dim <= 128 and any tile size; bf16 inputs
// with d in {64,128} and 128x128 tiles go to the tcgen05 kernels instead.
//
// Unlike the reference, the backward is deterministic: dQ is accumulated per
// query row (query-block-major walk over the CSR list) and dK/dV per key row
// (key-block-major walk over the transposed list), with no atomics.
#include "asa_internal.h"
#include <climits>

namespace asa {
namespace {

constexpr int KT = 32;      // keys staged per chunk
constexpr int QTHREADS = 128;

// ---------------------------------------------------------------------------
// τ / block mask.  One thread per query; the CTA's 128 queries stream every
// key (K staged 32 rows at a time in shared memory, read as broadcasts).
// Reference: build_mask_kernel :150-217.
// ---------------------------------------------------------------------------
// Smallest query position in query block qb (the reference's tile-load
// zeroing can only touch keys whose position exceeds it).
__device__ __forceinline__ int block_qmin(const Shape& sh, const int32_t* __restrict__ Qidx_bh,
                                          int qb, int* red) {
    int m = INT_MAX;
    for (int i = threadIdx.x; i < sh.BM && qb * sh.BM + i < sh.NQ; i += blockDim.x)
        m = min(m, Qidx_bh[qb * sh.BM + i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = min(m, __shfl_xor_sync(0xffffffffu, m, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    int r = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) r = min(r, red[w]);
    return r;
}

__device__ __forceinline__ int block_qmax(int v, int* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    int r = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) r = max(r, red[w]);
    return r;
}

// Threads per CTA for query-major kernels: the CTA covers (part of) one
// query block so all its queries share one tile list and one tile staging.
inline int qthreads(int BM) {
    int t = BM < QTHREADS ? BM : QTHREADS;
    return (t + 31) / 32 * 32;
}

// ---------------------------------------------------------------------------
// τ / block mask.  One thread per query; the CTA's queries (one query
// block, or a 128-query part of it) stream every key, K staged 32 rows at a
// time in shared memory and read as broadcasts.  The staging reproduces the
// reference's tile-load zeroing when sh.ref_load is set.
// Reference: build_mask_kernel :150-217.
// ---------------------------------------------------------------------------
template <typename T, int DM, int KM>
__global__ void __launch_bounds__(QTHREADS)
simt_tau_mask_kernel(Shape sh, const T* __restrict__ Q, const T* __restrict__ K,
                     const int32_t* __restrict__ Qidx, const int32_t* __restrict__ Kidx,
                     float* __restrict__ tau, uint8_t* __restrict__ M, float* __restrict__ topv,
                     int32_t* __restrict__ topi) {
    __shared__ float Ks[KT][DM];
    __shared__ int Kp[KT];
    __shared__ int red[QTHREADS / 32];
    const int QT = blockDim.x;
    const int tid = threadIdx.x;
    const int bh = blockIdx.y;
    const int subs = (sh.BM + QT - 1) / QT;
    const int qb = blockIdx.x / subs;
    const int inblk = (blockIdx.x % subs) * QT + tid;
    const int q = qb * sh.BM + inblk;
    const bool qv = inblk < sh.BM && q < sh.NQ;
    const int d = sh.d;
    const size_t qrow = (size_t)bh * sh.NQ + (qv ? q : 0);
    const int32_t* Qidx_bh = Qidx + (size_t)bh * sh.NQ;

    float qr[DM];
#pragma unroll
    for (int t = 0; t < DM; ++t) qr[t] = (qv && t < d) ? to_f(Q[qrow * d + t]) : 0.0f;
    const int qpos = !qv ? INT_MIN : (sh.causal ? Qidx[qrow] : INT_MAX);
    const int cta_max = block_qmax(qpos, red);
    const int qmin = sh.ref_load ? block_qmin(sh, Qidx_bh, qb, red) : INT_MAX;

    TopK<KM> tk;
    tk.init(sh.k);
    for (int start = 0; start < sh.NK; start += KT) {
        int any = 0;
        if (tid < KT) {
            const int kn = start + tid;
            const int kp = kn < sh.NK ? (sh.causal ? Kidx[(size_t)bh * sh.NK + kn] : INT_MIN) : INT_MAX;
            Kp[tid] = kp;
            any = (kn < sh.NK) && kp <= cta_max;
        }
        if (!__syncthreads_or(any)) continue;
        for (int x = tid; x < KT * DM; x += QT) {
            const int j = x / DM, t = x % DM, kn = start + j;
            bool ok = kn < sh.NK && t < d;
            if (ok && sh.ref_load && Kp[j] > qmin) ok = ref_keep(sh, Qidx_bh, qb, kn, t, Kp[j]);
            Ks[j][t] = ok ? to_f(K[((size_t)bh * sh.NK + kn) * d + t]) : 0.0f;
        }
        __syncthreads();
        if (qv) {
            for (int j = 0; j < KT; j += 2) {
                const int kn0 = start + j, kn1 = kn0 + 1;
                const bool v0 = kn0 < sh.NK && Kp[j] <= qpos;
                const bool v1 = kn1 < sh.NK && Kp[j + 1] <= qpos;
                if (!(v0 || v1)) continue;
                float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
                for (int t = 0; t < DM; ++t) {
                    if (t < d) {
                        a0 = __fmaf_rn(qr[t], Ks[j][t], a0);
                        a1 = __fmaf_rn(qr[t], Ks[j + 1][t], a1);
                    }
                }
                if (v0) {
                    const float s = clamp_score(a0, sh.scale);
                    if (s > tk.threshold()) tk.insert(s, kn0);
                }
                if (v1) {
                    const float s = clamp_score(a1, sh.scale);
                    if (s > tk.threshold()) tk.insert(s, kn1);
                }
            }
        }
        __syncthreads();
    }
    if (!qv) return;
    if (topv) {   // the row's top-k in order (score desc, key asc)
#pragma unroll
        for (int j = 0; j < KM; ++j)
            if (j >= KM - sh.k) {
                topv[qrow * sh.k + j - (KM - sh.k)] = tk.v[j];
                topi[qrow * sh.k + j - (KM - sh.k)] = tk.i[j];
            }
    }
    if (tau) tau[qrow] = ref_tau<KM>(tk.v, sh.k, sh.alpha);
    const size_t base = ((size_t)bh * sh.nQB + qb) * sh.nKB;
#pragma unroll
    for (int j = 0; j < KM; ++j)
        if (tk.i[j] >= 0) M[base + tk.i[j] / sh.BN] = 1;   // same-value writes, as :215
}


// ---------------------------------------------------------------------------
// Exact α-entmax threshold (asa_tau_mode ASA_TAU_EXACT): τ with
// Σ_j [(α-1)s_j - τ]_+^{1/(α-1)} = 1 over every visible key of the row.  One
// thread per query, kExactPasses passes over the keys: the first finds the
// row maximum s_max, which brackets τ in [(α-1)s_max - 1, (α-1)s_max]; each
// later pass evaluates F(τ) = Σ u_+^{1/(α-1)} and Σ u_+^{(2-α)/(α-1)} and
// takes a Newton step (F is convex and decreasing, so from the bracket's
// left end the steps climb monotonically), falling back to bisection when a
// step leaves the bracket.  The last pass also sets M for every tile that
// holds a positive weight at the bracket's left end, which bounds the final
// τ from below: a superset of the tiles the final τ leaves weight in.
// No counterpart in the reference (whose τ comes from the top-k only,
// :51-148); K is staged without the reference's tile-load zeroing.
// ---------------------------------------------------------------------------
template <typename T, int DM>
__global__ void __launch_bounds__(QTHREADS)
simt_exact_tau_kernel(Shape sh, const T* __restrict__ Q, const T* __restrict__ K,
                      const int32_t* __restrict__ Qidx, const int32_t* __restrict__ Kidx,
                      float* __restrict__ tau, uint8_t* __restrict__ M) {
    __shared__ float Ks[KT][DM];
    __shared__ int Kp[KT];
    __shared__ int red[QTHREADS / 32];
    const int QT = blockDim.x;
    const int tid = threadIdx.x;
    const int bh = blockIdx.y;
    const int subs = (sh.BM + QT - 1) / QT;
    const int qb = blockIdx.x / subs;
    const int inblk = (blockIdx.x % subs) * QT + tid;
    const int q = qb * sh.BM + inblk;
    const bool qv = inblk < sh.BM && q < sh.NQ;
    const int d = sh.d;
    const size_t qrow = (size_t)bh * sh.NQ + (qv ? q : 0);

    float qr[DM];
#pragma unroll
    for (int t = 0; t < DM; ++t) qr[t] = (qv && t < d) ? to_f(Q[qrow * d + t]) : 0.0f;
    const int qpos = !qv ? INT_MIN : (sh.causal ? Qidx[qrow] : INT_MAX);
    const int cta_max = block_qmax(qpos, red);
    const float inv = __fdiv_rn(1.0f, sh.am1);
    float smax = -INFINITY, tq = 0.0f, lo = 0.0f, hi = 0.0f;
    uint8_t* Mrow = M + ((size_t)bh * sh.nQB + qb) * sh.nKB;
    for (int pass = 0; pass < kExactPasses; ++pass) {
        const bool last = pass == kExactPasses - 1;
        float F = 0.0f, Dd = 0.0f;
        for (int start = 0; start < sh.NK; start += KT) {
            int any = 0;
            if (tid < KT) {
                const int kn = start + tid;
                const int kp = kn < sh.NK ? (sh.causal ? Kidx[(size_t)bh * sh.NK + kn] : INT_MIN) : INT_MAX;
                Kp[tid] = kp;
                any = (kn < sh.NK) && kp <= cta_max;
            }
            if (!__syncthreads_or(any)) continue;
            for (int x = tid; x < KT * DM; x += QT) {
                const int j = x / DM, t = x % DM, kn = start + j;
                Ks[j][t] = (kn < sh.NK && t < d) ? to_f(K[((size_t)bh * sh.NK + kn) * d + t]) : 0.0f;
            }
            __syncthreads();
            if (qv) {
                for (int j = 0; j < KT; ++j) {
                    const int kn = start + j;
                    if (kn >= sh.NK || !(Kp[j] <= qpos)) continue;
                    float a = 0.0f;
#pragma unroll
                    for (int t = 0; t < DM; ++t)
                        if (t < d) a = __fmaf_rn(qr[t], Ks[j][t], a);
                    const float sc = clamp_score(a, sh.scale);
                    if (pass == 0) { smax = fmaxf(smax, sc); continue; }
                    const float u = __fmaf_rn(sh.am1, sc, -tq);
                    if (u > 0.0f) {
                        const float p = pow_exact(u, sh.pinv), w = pow_exact(u, sh.pe2);
                        if (isfinite(p)) F += p;
                        if (isfinite(w)) Dd += w;
                    }
                    if (last && __fmaf_rn(sh.am1, sc, -lo) > 0.0f) Mrow[kn / sh.BN] = 1;
                }
            }
            __syncthreads();
        }
        if (pass == 0) {
            if (!(smax > -INFINITY)) smax = 0.0f;     // no visible key: no weight anywhere
            hi = __fmul_rn(sh.am1, smax);
            lo = __fadd_rn(hi, -1.0f);
            tq = lo;
            continue;
        }
        const float g = F - 1.0f;
        if (g >= 0.0f) lo = tq; else hi = tq;
        float tn = (Dd > 0.0f) ? tq + g / (inv * Dd) : tq;
        if (!(tn >= lo && tn <= hi)) tn = 0.5f * (lo + hi);
        tq = tn;
    }
    if (qv) tau[qrow] = tq;
}

// ---------------------------------------------------------------------------
// Query-major walk over a query block's active tiles (CSR order, keys
// ascending), shared by the forward (MODE 0), the backward's row statistics
// (MODE 1), dQ (MODE 2) and the row statistics of the Jacobian gradient
// (MODE 3: accdO = (n + EPS)·Σ_j w_j (v_j·dO) / Σ_j w_j with
// w = u^{(2-α)/(α-1)}, so that dQ/dK/dV's "accdO·invN" term becomes the
// w-weighted mean of v·dO).  Each thread owns one query row; its q (and dO)
// row sits in padded shared memory, K/V chunks are read as broadcasts.
// References: splash_forward_sparse :244-341, splash_backward_sparse pass 1
// :395-437 and pass 2's dQ part :439-534.
// ---------------------------------------------------------------------------
template <typename T, typename TO, int DM, int MODE>
__global__ void __launch_bounds__(QTHREADS)
simt_rows_kernel(Shape sh, const T* __restrict__ Q, const T* __restrict__ K,
                 const T* __restrict__ V, const int32_t* __restrict__ Qidx,
                 const int32_t* __restrict__ Kidx, const float* __restrict__ tau,
                 const int32_t* __restrict__ ptr, const int32_t* __restrict__ idx,
                 const T* __restrict__ dO, const float* __restrict__ invN_in,
                 const float* __restrict__ accdO_in, TO* __restrict__ out,
                 float* __restrict__ out32, float* __restrict__ r0, float* __restrict__ r1) {
    extern __shared__ float smem[];
    const int QT = blockDim.x;
    const int tid = threadIdx.x;
    const int bh = blockIdx.y;
    const int subs = (sh.BM + QT - 1) / QT;
    const int qb = blockIdx.x / subs;
    const int inblk = (blockIdx.x % subs) * QT + tid;
    const int q = qb * sh.BM + inblk;
    const bool qv = inblk < sh.BM && q < sh.NQ;
    const int d = sh.d;
    const size_t qrow = (size_t)bh * sh.NQ + (qv ? q : 0);
    constexpr int LD = DM + 1;
    float* qs = smem;                          // [QT][DM+1]
    constexpr bool kDO = MODE >= 2;            // dO rows staged (MODE 2 and 3)
    float* gs_ = qs + QT * LD;                 // [QT][DM+1] dO rows
    float* Ks = gs_ + (kDO ? QT * LD : 0);
    float* Vs = Ks + KT * DM;
    __shared__ int Kp[KT];
    __shared__ int red[QTHREADS / 32];
    const int32_t* Qidx_bh = Qidx + (size_t)bh * sh.NQ;
    const int qmin = sh.ref_load ? block_qmin(sh, Qidx_bh, qb, red) : INT_MAX;

    for (int t = 0; t < DM; ++t) {
        qs[tid * LD + t] = (qv && t < d) ? to_f(Q[qrow * d + t]) : 0.0f;
        if (kDO) gs_[tid * LD + t] = (qv && t < d) ? to_f(dO[qrow * d + t]) : 0.0f;
    }
    const int qpos = !qv ? INT_MIN : (sh.causal ? Qidx[qrow] : INT_MAX);
    const float tq = qv ? tau[qrow] : 0.0f;
    float invN = 0.0f, accdO = 0.0f;
    if (MODE == 2 && qv) { invN = invN_in[qrow]; accdO = accdO_in[qrow]; }
    const float minv2 = __fmul_rn(-invN, invN);

    float acc[DM];
#pragma unroll
    for (int t = 0; t < DM; ++t) acc[t] = 0.0f;
    float n = 0.0f;
    float wA = 0.0f, wB = 0.0f;                // MODE 3: Σ w·(v·dO), Σ w

    const int32_t* p = ptr + (size_t)bh * (sh.nQB + 1);
    const int32_t* ix = idx + (size_t)bh * sh.nQB * sh.nKB;
    const int e0 = p[qb], e1 = p[qb + 1];
    for (int e = e0; e < e1; ++e) {
        const int start = ix[e] * sh.BN;
        for (int c0 = 0; c0 < sh.BN; c0 += KT) {
            const int cn = min(KT, sh.BN - c0);
            __syncthreads();
            if (tid < KT) {
                const int kn = start + c0 + tid;
                Kp[tid] = (tid < cn && kn < sh.NK)
                              ? (sh.causal ? Kidx[(size_t)bh * sh.NK + kn] : INT_MIN) : INT_MAX;
            }
            __syncthreads();
            for (int x = tid; x < KT * DM; x += QT) {
                const int j = x / DM, t = x % DM, kn = start + c0 + j;
                bool ok = j < cn && kn < sh.NK && t < d;
                if (ok && sh.ref_load && Kp[j] > qmin) ok = ref_keep(sh, Qidx_bh, qb, kn, t, Kp[j]);
                const size_t off = ((size_t)bh * sh.NK + kn) * d + t;
                Ks[j * DM + t] = ok ? to_f(K[off]) : 0.0f;
                Vs[j * DM + t] = ok ? to_f(V[off]) : 0.0f;
            }
            __syncthreads();
            if (!qv) continue;
            for (int j = 0; j < cn; ++j) {
                if (start + c0 + j >= sh.NK || !(Kp[j] <= qpos)) continue;
                float a = 0.0f;
#pragma unroll
                for (int t = 0; t < DM; ++t)
                    if (t < d) a = __fmaf_rn(qs[tid * LD + t], Ks[j * DM + t], a);
                const float s = clamp_score(a, sh.scale);
                float u;
                const float pr = entmax_p(s, sh.am1, tq, sh.pinv, &u);
                if (MODE == 3) {
                    n = __fadd_rn(n, pr);
                    if (u > ASA_EPS) {
                        const float w = pow_exact(fmaxf(u, ASA_EPS), sh.pe2);
                        if (isfinite(w)) {
                            float vd = 0.0f;
#pragma unroll
                            for (int t = 0; t < DM; ++t)
                                if (t < d) vd = __fmaf_rn(Vs[j * DM + t], gs_[tid * LD + t], vd);
                            wA = __fmaf_rn(w, vd, wA);
                            wB = __fadd_rn(wB, w);
                        }
                    }
                } else if (MODE != 2) {
                    n = __fadd_rn(n, pr);
#pragma unroll
                    for (int t = 0; t < DM; ++t)
                        if (t < d) acc[t] = __fmaf_rn(pr, Vs[j * DM + t], acc[t]);
                } else {
                    // dp = Σ_t v_t·dO_t·invN + (acc·dO)·(-invN²)  (:481-491)
                    float dp = 0.0f;
#pragma unroll
                    for (int t = 0; t < DM; ++t)
                        if (t < d) dp = __fmaf_rn(__fmul_rn(Vs[j * DM + t], gs_[tid * LD + t]), invN, dp);
                    dp = __fmaf_rn(accdO, minv2, dp);
                    float gu = 0.0f;
                    if (u > ASA_EPS && fabsf(sh.am1) > ASA_EPS) {          // :494-501
                        const float pw = pow_exact(fmaxf(u, ASA_EPS), sh.pe2);
                        if (isfinite(pw)) gu = __fmul_rn(__fmul_rn(sh.inv_am1b, pw), dp);
                    }
                    float g = __fmul_rn(gu, sh.am1);                       // :503-507
                    if (!isfinite(g)) g = 0.0f;
#pragma unroll
                    for (int t = 0; t < DM; ++t) {                          // :509-514
                        if (t < d) {
                            const float c = __fmul_rn(__fmul_rn(g, Ks[j * DM + t]), sh.scale);
                            if (isfinite(c)) acc[t] = __fadd_rn(acc[t], c);
                        }
                    }
                }
            }
        }
    }
    if (!qv) return;
    if (MODE == 0) {
        const float inv = __fdiv_rn(1.0f, __fadd_rn(n, ASA_EPS));          // :328
#pragma unroll
        for (int t = 0; t < DM; ++t) {
            if (t < d) {
                float o = __fmul_rn(acc[t], inv);
                if (!isfinite(o)) o = 0.0f;                                // :335-337
                out[qrow * d + t] = from_f<TO>(o);
                if (out32) out32[qrow * d + t] = o;
            }
        }
        if (r0) r0[qrow] = n;
    } else if (MODE == 1) {
        float ad = 0.0f;
#pragma unroll
        for (int t = 0; t < DM; ++t)
            if (t < d) ad = __fmaf_rn(acc[t], to_f(dO[qrow * d + t]), ad);  // :487-490
        r0[qrow] = __fdiv_rn(1.0f, __fadd_rn(n, ASA_EPS));                 // :435
        r1[qrow] = ad;
    } else if (MODE == 3) {
        const float np = __fadd_rn(n, ASA_EPS);
        r0[qrow] = __fdiv_rn(1.0f, np);
        r1[qrow] = wB > 0.0f ? __fmul_rn(__fdiv_rn(wA, wB), np) : 0.0f;
    } else {
#pragma unroll
        for (int t = 0; t < DM; ++t) {
            if (t < d) {
                float v = acc[t];
                if (!isfinite(v)) v = 0.0f;                                // :529-531
                out[qrow * d + t] = from_f<TO>(v);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Key-major walk for dK / dV: each thread owns one key row and visits, in
// ascending order, every query of every query block whose tile list holds
// this key block.  Pair arithmetic is the reference's (:463-519); sums run
// in query order, so the result is deterministic.
// ---------------------------------------------------------------------------
template <typename T, typename TO, int DM, bool DO_DK, bool DO_DV>
__global__ void __launch_bounds__(QTHREADS)
simt_dkdv_kernel(Shape sh, const T* __restrict__ Q, const T* __restrict__ K,
                 const T* __restrict__ V, const int32_t* __restrict__ Qidx,
                 const int32_t* __restrict__ Kidx, const float* __restrict__ tau,
                 const int32_t* __restrict__ cptr, const int32_t* __restrict__ cidx,
                 const T* __restrict__ dO, const float* __restrict__ invN_in,
                 const float* __restrict__ accdO_in, TO* __restrict__ dK, TO* __restrict__ dV) {
    extern __shared__ float smem[];
    constexpr int QC = 32;
    constexpr int LD = DM + 1;
    const int KTH = blockDim.x;
    const int tid = threadIdx.x;
    const int bh = blockIdx.y;
    const int subs = (sh.BN + KTH - 1) / KTH;
    const int kb = blockIdx.x / subs;
    const int inblk = (blockIdx.x % subs) * KTH + tid;
    const int kn = kb * sh.BN + inblk;
    const bool kv = inblk < sh.BN && kn < sh.NK;
    const int d = sh.d;
    const size_t krow = (size_t)bh * sh.NK + (kv ? kn : 0);
    float* ks = smem;               // [KTH][LD]
    float* vs = ks + KTH * LD;      // [KTH][LD]
    float* Qc = vs + KTH * LD;      // [QC][DM]
    float* Gc = Qc + QC * DM;       // [QC][DM]
    __shared__ float tq_s[QC], in_s[QC], ad_s[QC];
    __shared__ int qp_s[QC];
    __shared__ int red[QTHREADS / 32];

    for (int t = 0; t < DM; ++t) {
        ks[tid * LD + t] = (kv && t < d) ? to_f(K[krow * d + t]) : 0.0f;
        vs[tid * LD + t] = (kv && t < d) ? to_f(V[krow * d + t]) : 0.0f;
    }
    const int kpos = !kv ? INT_MAX : (sh.causal ? Kidx[krow] : INT_MIN);
    float dk[DO_DK ? DM : 1], dv[DO_DV ? DM : 1];
#pragma unroll
    for (int t = 0; t < DM; ++t) {
        if constexpr (DO_DK) dk[t] = 0.0f;
        if constexpr (DO_DV) dv[t] = 0.0f;
    }
    const int32_t* cp = cptr + (size_t)bh * (sh.nKB + 1);
    const int32_t* cx = cidx + (size_t)bh * sh.nKB * sh.nQB;
    const int e0 = cp[kb], e1 = cp[kb + 1];
    const int32_t* Qidx_bh = Qidx + (size_t)bh * sh.NQ;
    bool dirty = false;
    for (int e = e0; e < e1; ++e) {
        const int qb = cx[e];
        // rows as the consumers of query block qb see them (reference tile-load
        // zeroing); rebuilt only when this key can be touched by it
        const int qmin = sh.ref_load ? block_qmin(sh, Qidx_bh, qb, red) : INT_MAX;
        if (kv) {
            const bool need = sh.ref_load && kpos > qmin;
            if (need || dirty) {
                for (int t = 0; t < DM; ++t) {
                    const bool keep = t < d && (!need || ref_keep(sh, Qidx_bh, qb, kn, t, kpos));
                    ks[tid * LD + t] = keep ? to_f(K[krow * d + t]) : 0.0f;
                    vs[tid * LD + t] = keep ? to_f(V[krow * d + t]) : 0.0f;
                }
                dirty = need;
            }
        }
        const int q0 = qb * sh.BM;
        const int qend = min(q0 + sh.BM, sh.NQ);
        for (int c0 = q0; c0 < qend; c0 += QC) {
            const int cn = min(QC, qend - c0);
            __syncthreads();
            for (int x = tid; x < QC * DM; x += KTH) {
                const int j = x / DM, t = x % DM;
                const bool ok = j < cn && t < d;
                const size_t off = ((size_t)bh * sh.NQ + c0 + j) * d + t;
                Qc[j * DM + t] = ok ? to_f(Q[off]) : 0.0f;
                Gc[j * DM + t] = ok ? to_f(dO[off]) : 0.0f;
            }
            if (tid < QC) {
                const bool ok = tid < cn;
                const size_t r = (size_t)bh * sh.NQ + c0 + (ok ? tid : 0);
                tq_s[tid] = ok ? tau[r] : 0.0f;
                in_s[tid] = ok ? invN_in[r] : 0.0f;
                ad_s[tid] = ok ? accdO_in[r] : 0.0f;
                qp_s[tid] = ok ? (sh.causal ? Qidx[r] : INT_MAX) : INT_MIN;
            }
            __syncthreads();
            if (!kv) continue;
            for (int j = 0; j < cn; ++j) {
                if (!(kpos <= qp_s[j])) continue;
                float a = 0.0f;
#pragma unroll
                for (int t = 0; t < DM; ++t)
                    if (t < d) a = __fmaf_rn(Qc[j * DM + t], ks[tid * LD + t], a);
                const float s = clamp_score(a, sh.scale);
                float u;
                const float pr = entmax_p(s, sh.am1, tq_s[j], sh.pinv, &u);
                const float invN = in_s[j];
                if constexpr (DO_DV) {
                    const float pb = __fmul_rn(pr, invN);                   // :471
#pragma unroll
                    for (int t = 0; t < DM; ++t) {
                        if (t < d) {
                            const float c = __fmul_rn(pb, Gc[j * DM + t]);
                            if (isfinite(c)) dv[t] = __fadd_rn(dv[t], c);
                        }
                    }
                }
                if constexpr (DO_DK) {
                    float dp = 0.0f;
#pragma unroll
                    for (int t = 0; t < DM; ++t)
                        if (t < d) dp = __fmaf_rn(__fmul_rn(vs[tid * LD + t], Gc[j * DM + t]), invN, dp);
                    dp = __fmaf_rn(ad_s[j], __fmul_rn(-invN, invN), dp);
                    float gu = 0.0f;
                    if (u > ASA_EPS && fabsf(sh.am1) > ASA_EPS) {
                        const float pw = pow_exact(fmaxf(u, ASA_EPS), sh.pe2);
                        if (isfinite(pw)) gu = __fmul_rn(__fmul_rn(sh.inv_am1b, pw), dp);
                    }
                    float g = __fmul_rn(gu, sh.am1);
                    if (!isfinite(g)) g = 0.0f;
#pragma unroll
                    for (int t = 0; t < DM; ++t) {                          // :516-519
                        if (t < d) {
                            const float c = __fmul_rn(__fmul_rn(g, Qc[j * DM + t]), sh.scale);
                            if (isfinite(c)) dk[t] = __fadd_rn(dk[t], c);
                        }
                    }
                }
            }
        }
    }
    if (!kv) return;
#pragma unroll
    for (int t = 0; t < DM; ++t) {
        if (t < d) {
            if constexpr (DO_DK) dK[krow * d + t] = from_f<TO>(dk[t]);
            if constexpr (DO_DV) dV[krow * d + t] = from_f<TO>(dv[t]);
        }
    }
}

template <typename F>
cudaError_t set_smem(F* f, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

// dtype dispatch helpers -----------------------------------------------------
#define ASA_DISPATCH_T(dt, T, ...)                                                  \
    do {                                                                            \
        if ((dt) == ASA_DTYPE_F32) { using T = float; __VA_ARGS__; }                \
        else { using T = __nv_bfloat16; __VA_ARGS__; }                              \
    } while (0)
#define ASA_DISPATCH_DM(dval, DMV, ...)                                             \
    do {                                                                            \
        if ((dval) <= 64) { constexpr int DMV = 64; __VA_ARGS__; }                  \
        else { constexpr int DMV = 128; __VA_ARGS__; }                              \
    } while (0)

template <typename T, int DM, int KM>
cudaError_t launch_tau_mask(const Shape& s, const void* Q, const void* K, const int32_t* Qidx,
                            const int32_t* Kidx, float* tau, uint8_t* M, float* topv, int32_t* topi,
                            cudaStream_t st) {
    const int QT = qthreads(s.BM);
    dim3 grid(s.nQB * ((s.BM + QT - 1) / QT), s.BH);
    simt_tau_mask_kernel<T, DM, KM><<<grid, QT, 0, st>>>(
        s, (const T*)Q, (const T*)K, Qidx, Kidx, tau, M, topv, topi);
    note_launch();
    return cudaGetLastError();
}

template <typename T, typename TO, int DM, int MODE>
cudaError_t launch_rows(const Shape& s, const void* Q, const void* K, const void* V,
                        const int32_t* Qidx, const int32_t* Kidx, const float* tau,
                        const int32_t* ptr, const int32_t* idx, const void* dO,
                        const float* invN, const float* accdO, void* out, float* out32,
                        float* r0, float* r1, cudaStream_t st) {
    const int QT = qthreads(s.BM);
    const int subs = (s.BM + QT - 1) / QT;
    const size_t smem = sizeof(float) * ((size_t)QT * (DM + 1) * (MODE >= 2 ? 2 : 1) + 2 * KT * DM);
    auto kern = simt_rows_kernel<T, TO, DM, MODE>;
    cudaError_t e = set_smem(kern, smem);
    if (e != cudaSuccess) return e;
    dim3 grid(s.nQB * subs, s.BH);
    kern<<<grid, QT, smem, st>>>(s, (const T*)Q, (const T*)K, (const T*)V, Qidx, Kidx, tau, ptr,
                                 idx, (const T*)dO, invN, accdO, (TO*)out, out32, r0, r1);
    note_launch();
    return cudaGetLastError();
}

template <typename T, typename TO, int DM, bool DK, bool DV>
cudaError_t launch_dkdv(const Shape& s, const void* Q, const void* K, const void* V,
                        const int32_t* Qidx, const int32_t* Kidx, const float* tau,
                        const int32_t* cptr, const int32_t* cidx, const void* dO,
                        const float* invN, const float* accdO, void* dK, void* dV,
                        cudaStream_t st) {
    const int KTH = qthreads(s.BN);
    const int subs = (s.BN + KTH - 1) / KTH;
    const size_t smem = sizeof(float) * ((size_t)2 * KTH * (DM + 1) + 2 * 32 * DM);
    auto kern = simt_dkdv_kernel<T, TO, DM, DK, DV>;
    cudaError_t e = set_smem(kern, smem);
    if (e != cudaSuccess) return e;
    dim3 grid(s.nKB * subs, s.BH);
    kern<<<grid, KTH, smem, st>>>(s, (const T*)Q, (const T*)K, (const T*)V, Qidx, Kidx, tau, cptr,
                                  cidx, (const T*)dO, invN, accdO, (TO*)dK, (TO*)dV);
    note_launch();
    return cudaGetLastError();
}

}  // namespace

cudaError_t simt_tau_mask(const Shape& s, const void* Q, const void* K, const int32_t* Qidx,
                          const int32_t* Kidx, float* tau, uint8_t* M, cudaStream_t st, float* topv,
                          int32_t* topi) {
    cudaError_t e = cudaMemsetAsync(M, 0, (size_t)s.BH * s.nQB * s.nKB, st);
    if (e != cudaSuccess) return e;
    ASA_DISPATCH_T(s.in_dtype, T, ASA_DISPATCH_DM(s.d, DM, {
        if (s.k <= 8) return launch_tau_mask<T, DM, 8>(s, Q, K, Qidx, Kidx, tau, M, topv, topi, st);
        if (s.k <= 16) return launch_tau_mask<T, DM, 16>(s, Q, K, Qidx, Kidx, tau, M, topv, topi, st);
        return launch_tau_mask<T, DM, 32>(s, Q, K, Qidx, Kidx, tau, M, topv, topi, st);
    }));
    return cudaErrorInvalidValue;
}

cudaError_t simt_forward(const Shape& s, const void* Q, const void* K, const void* V,
                         const int32_t* Qidx, const int32_t* Kidx, const float* tau,
                         const int32_t* ptr, const int32_t* idx, void* O, float* O32,
                         float* rownorm, cudaStream_t st) {
    ASA_DISPATCH_T(s.in_dtype, T, ASA_DISPATCH_T(s.out_dtype, TO, ASA_DISPATCH_DM(s.d, DM, {
        return launch_rows<T, TO, DM, 0>(s, Q, K, V, Qidx, Kidx, tau, ptr, idx, nullptr, nullptr,
                                         nullptr, O, O32, rownorm, nullptr, st);
    })));
    return cudaErrorInvalidValue;
}

cudaError_t simt_rowstats(const Shape& s, const void* Q, const void* K, const void* V,
                          const int32_t* Qidx, const int32_t* Kidx, const float* tau,
                          const int32_t* ptr, const int32_t* idx, const void* dO,
                          float* invN, float* accdO, cudaStream_t st) {
    ASA_DISPATCH_T(s.in_dtype, T, ASA_DISPATCH_DM(s.d, DM, {
        return launch_rows<T, float, DM, 1>(s, Q, K, V, Qidx, Kidx, tau, ptr, idx, dO, nullptr,
                                            nullptr, nullptr, nullptr, invN, accdO, st);
    }));
    return cudaErrorInvalidValue;
}

cudaError_t simt_exact_tau(const Shape& s, const void* Q, const void* K, const int32_t* Qidx,
                           const int32_t* Kidx, float* tau, uint8_t* M, cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(M, 0, (size_t)s.BH * s.nQB * s.nKB, st);
    if (e != cudaSuccess) return e;
    ASA_DISPATCH_T(s.in_dtype, T, ASA_DISPATCH_DM(s.d, DM, {
        const int QT = qthreads(s.BM);
        dim3 grid(s.nQB * ((s.BM + QT - 1) / QT), s.BH);
        simt_exact_tau_kernel<T, DM><<<grid, QT, 0, st>>>(s, (const T*)Q, (const T*)K, Qidx, Kidx, tau, M);
        note_launch();
        return cudaGetLastError();
    }));
    return cudaErrorInvalidValue;
}

cudaError_t simt_jacobian_stats(const Shape& s, const void* Q, const void* K, const void* V,
                                const int32_t* Qidx, const int32_t* Kidx, const float* tau,
                                const int32_t* ptr, const int32_t* idx, const void* dO,
                                float* invN, float* accdO, cudaStream_t st) {
    ASA_DISPATCH_T(s.in_dtype, T, ASA_DISPATCH_DM(s.d, DM, {
        return launch_rows<T, float, DM, 3>(s, Q, K, V, Qidx, Kidx, tau, ptr, idx, dO, nullptr,
                                            nullptr, nullptr, nullptr, invN, accdO, st);
    }));
    return cudaErrorInvalidValue;
}

cudaError_t simt_dq(const Shape& s, const void* Q, const void* K, const void* V,
                    const int32_t* Qidx, const int32_t* Kidx, const float* tau,
                    const int32_t* ptr, const int32_t* idx, const void* dO,
                    const float* invN, const float* accdO, void* dQ, cudaStream_t st) {
    ASA_DISPATCH_T(s.in_dtype, T, ASA_DISPATCH_T(s.out_dtype, TO, ASA_DISPATCH_DM(s.d, DM, {
        return launch_rows<T, TO, DM, 2>(s, Q, K, V, Qidx, Kidx, tau, ptr, idx, dO, invN, accdO,
                                         dQ, nullptr, nullptr, nullptr, st);
    })));
    return cudaErrorInvalidValue;
}

cudaError_t simt_dkdv(const Shape& s, const void* Q, const void* K, const void* V,
                      const int32_t* Qidx, const int32_t* Kidx, const float* tau,
                      const int32_t* cptr, const int32_t* cidx, const void* dO,
                      const float* invN, const float* accdO, void* dK, void* dV,
                      cudaStream_t st) {
    ASA_DISPATCH_T(s.in_dtype, T, ASA_DISPATCH_T(s.out_dtype, TO, {
        if (s.d <= 64)
            return launch_dkdv<T, TO, 64, true, true>(s, Q, K, V, Qidx, Kidx, tau, cptr, cidx, dO,
                                                      invN, accdO, dK, dV, st);
        // d > 64: dK and dV in two passes so each keeps one 128-wide accumulator
        cudaError_t e = launch_dkdv<T, TO, 128, true, false>(s, Q, K, V, Qidx, Kidx, tau, cptr,
                                                             cidx, dO, invN, accdO, dK, dV, st);
        if (e != cudaSuccess) return e;
        return launch_dkdv<T, TO, 128, false, true>(s, Q, K, V, Qidx, Kidx, tau, cptr, cidx, dO,
                                                    invN, accdO, dK, dV, st);
    }));
    return cudaErrorInvalidValue;
}

}  // namespace asa
