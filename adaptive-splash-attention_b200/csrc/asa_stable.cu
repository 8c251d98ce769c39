// asa_stable.cu -- the top-k-only ("stable") α-entmax operator.
//
// Reference: the "stable" kernel of AdaSplashNotebook.ipynb (notebook file
// lines 303-450: stable_entmax_threshold, stable_splash_kernel,
// stable_forward, stable_backward).  Per query it keeps the top-k clamped
// scores of the visible keys (the same strict-'>' top-k as the main
// operator: the engine's τ/mask kernels produce it, without tile-load
// zeroing), finds τ by five bisection steps, normalises the weights and
// returns O = Σ_j w_j V[key_j].  The notebook's backward returns zeros; this
// one is the operator's gradient.
//
// Gradient.  The bisection's steps are comparisons, so almost everywhere τ is
// an affine function of its starting bracket: τ = c_min·lo_0 + c_max·hi_0
// with lo_0 = (α-1)s_min - 1, hi_0 = (α-1)s_max + 1 (or the τ clamp's bound)
// and c_min + c_max = 1.  The forward records c_max, so dτ/ds_max =
// (α-1)c_max and dτ/ds_min = (α-1)c_min.  With p̃_j = u_j^{1/(α-1)} (u > EPS),
// N = max(Σ p̃, EPS), w_j = p̃_j / N, g_j = dO·V[key_j] and
// h_j = (g_j - Σ_i w_i g_i)/N (h_j = g_j/EPS when the EPS floor is active):
//   dL/ds_i = h_i ω_i - t_i Σ_j h_j ω_j,  ω_j = u_j^{(2-α)/(α-1)},
// with t_0 = c_max, t_{k-1} = c_min (else 0); a clamped score (|s| = 10)
// passes no gradient; dL/d(raw) = dL/ds · sm_scale.  Then
//   dQ_q = Σ_i dL/draw_i K[key_i],  dK[key_i] += dL/draw_i q,
//   dV[key_i] += w_i dO_q
// (dK and dV gather from many queries: fp32 atomics into an fp32 buffer,
// converted at the end; their last bits depend on the order of arrival, as
// the reference's own atomics-based backward does).
#include "asa_internal.h"

namespace asa {
namespace {

constexpr int STABLE_WARPS = 4;   // rows per CTA (one warp per row)

// The notebook's α clamp for this operator: [1.01, 3].
__host__ __device__ inline float stable_alpha(float a) { return fmaxf(1.01f, fminf(a, 3.0f)); }

// τ by the notebook's five bisection steps over the sorted scores s[0..k);
// returns τ and, through cmax, the weight of hi_0 (or of the upper clamp) in
// the final τ.
__device__ float stable_tau(const float* s, int k, float alpha, float* cmax) {
    const float am1 = __fadd_rn(alpha, -1.0f);
    const float inv = __fdiv_rn(1.0f, am1);
    const float s_max = s[0], s_min = s[k - 1];
    float lo = __fmaf_rn(am1, s_min, -1.0f), hi = __fmaf_rn(am1, s_max, 1.0f);
    float clo = 0.0f, chi = 1.0f;             // weights of hi_0 in lo and hi
    float tau = __fmul_rn(0.5f, __fadd_rn(lo, hi));
    float ct = 0.5f;
    for (int it = 0; it < ASA_HALLEY_ITERS; ++it) {
        float f = -1.0f;
        for (int j = 0; j < k; ++j) {
            const float u = __fmaf_rn(am1, s[j], -tau);
            if (u <= 0.0f) break;
            float up = powf(fmaxf(u, ASA_EPS), inv);
            if (!isfinite(up)) up = 0.0f;
            f = __fadd_rn(f, up);
        }
        if (fabsf(f) < 1e-4f) break;
        if (f > 0.0f) { lo = tau; clo = ct; } else { hi = tau; chi = ct; }
        tau = __fmul_rn(0.5f, __fadd_rn(lo, hi));
        ct = 0.5f * (clo + chi);
        const float tmin = __fmaf_rn(s_min, am1, -10.0f), tmax = __fmaf_rn(s_max, am1, 10.0f);
        if (tau < tmin) { tau = tmin; ct = 0.0f; }
        if (tau > tmax) { tau = tmax; ct = 1.0f; }
    }
    *cmax = ct;
    return tau;
}

// One warp per row: lane j < k holds entry j.
template <typename T, typename TO>
__global__ void __launch_bounds__(32 * STABLE_WARPS)
stable_fwd_kernel(Shape sh, float alpha, const T* __restrict__ V, const float* __restrict__ topv,
                  const int32_t* __restrict__ topi, TO* __restrict__ O, float* __restrict__ tau_out,
                  float* __restrict__ weights, float* __restrict__ tau_coef) {
    const size_t row = (size_t)blockIdx.x * STABLE_WARPS + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const size_t rows = (size_t)sh.BH * sh.NQ;
    if (row >= rows) return;
    const int k = sh.k, d = sh.d;
    const size_t bh = row / sh.NQ;
    float s[32];
    float w_mine = 0.0f;
    int key_mine = -1;
    if (lane == 0) {
        for (int j = 0; j < k; ++j) s[j] = topv[row * k + j];
        float cmax;
        const float am1 = __fadd_rn(alpha, -1.0f);
        const float inv = __fdiv_rn(1.0f, am1);
        const float tq = stable_tau(s, k, alpha, &cmax);
        float norm = 0.0f;
        for (int j = 0; j < k; ++j) {
            const float u = __fmaf_rn(am1, s[j], -tq);
            float pj = u > ASA_EPS ? powf(u, inv) : 0.0f;
            if (!isfinite(pj)) pj = 0.0f;
            s[j] = pj;
            norm = __fadd_rn(norm, pj);
        }
        norm = fmaxf(norm, ASA_EPS);
        for (int j = 0; j < k; ++j) {
            float pj = __fdiv_rn(s[j], norm);
            if (!isfinite(pj)) pj = __fdiv_rn(1.0f, (float)k);   // the notebook's fallback
            s[j] = pj;
            weights[row * k + j] = pj;
        }
        tau_out[row] = tq;
        tau_coef[row] = cmax;
    }
    __syncwarp();
    if (lane < k) {
        w_mine = weights[row * k + lane];
        key_mine = topi[row * k + lane];
    }
    // O[t] = Σ_j w_j V[key_j][t], the j-ordered FMA chain of the notebook
    for (int t = lane; t < d; t += 32) {
        float acc = 0.0f;
        for (int j = 0; j < k; ++j) {
            const float wj = __shfl_sync(0xffffffffu, w_mine, j);
            const int kj = __shfl_sync(0xffffffffu, key_mine, j);
            if (kj >= 0) acc = __fmaf_rn(wj, to_f(V[(bh * sh.NK + kj) * d + t]), acc);
        }
        if (!isfinite(acc)) acc = 0.0f;
        O[row * d + t] = from_f<TO>(acc);
    }
}

template <typename T, typename TO>
__global__ void __launch_bounds__(32 * STABLE_WARPS)
stable_bwd_kernel(Shape sh, float alpha, const T* __restrict__ Q, const T* __restrict__ K,
                  const T* __restrict__ V, const T* __restrict__ dO, const float* __restrict__ topv,
                  const int32_t* __restrict__ topi, const float* __restrict__ weights,
                  const float* __restrict__ tau, const float* __restrict__ tau_coef,
                  TO* __restrict__ dQ, float* __restrict__ dK32, float* __restrict__ dV32) {
    const size_t row = (size_t)blockIdx.x * STABLE_WARPS + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const size_t rows = (size_t)sh.BH * sh.NQ;
    if (row >= rows) return;
    const int k = sh.k, d = sh.d;
    const size_t bh = row / sh.NQ;
    const float am1 = alpha - 1.0f;
    const float inv = 1.0f / am1, e2 = (2.0f - alpha) * inv;
    const float tq = tau[row], cmax = tau_coef[row];
    // this lane's entry
    const bool has = lane < k;
    const int key = has ? topi[row * k + lane] : -1;
    const float sj = has ? topv[row * k + lane] : 0.0f;
    const float wj = has ? weights[row * k + lane] : 0.0f;
    const bool live = key >= 0;
    // g_j = dO·V[key_j]: one warp-wide dot per entry
    float gj = 0.0f;
    for (int j = 0; j < k; ++j) {
        const int kj = __shfl_sync(0xffffffffu, key, j);
        float part = 0.0f;
        if (kj >= 0)
            for (int t = lane; t < d; t += 32)
                part = fmaf(to_f(dO[row * d + t]), to_f(V[(bh * sh.NK + kj) * d + t]), part);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if (lane == j) gj = part;
    }
    // p̃_j, ω_j and N from the scores and τ, as the forward formed them
    const float u = __fmaf_rn(__fadd_rn(alpha, -1.0f), sj, -tq);
    float pt = (live && u > ASA_EPS) ? powf(u, inv) : 0.0f;
    if (!isfinite(pt)) pt = 0.0f;
    float om = (live && u > ASA_EPS) ? powf(u, e2) : 0.0f;
    if (!isfinite(om)) om = 0.0f;
    float N = pt, wg = live ? wj * gj : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        N += __shfl_xor_sync(0xffffffffu, N, o);
        wg += __shfl_xor_sync(0xffffffffu, wg, o);
    }
    const bool floor = !(N >= ASA_EPS);
    const float Nf = floor ? ASA_EPS : N;
    const float h = live ? (floor ? gj / Nf : (gj - wg) / Nf) : 0.0f;
    float hw = h * om;
    float sum_hw = hw;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum_hw += __shfl_xor_sync(0xffffffffu, sum_hw, o);
    float t_i = 0.0f;
    if (lane == 0) t_i += cmax;
    if (lane == k - 1) t_i += 1.0f - cmax;
    float ds = hw - t_i * sum_hw;
    if (!live || !(fabsf(sj) < 10.0f) || !isfinite(ds)) ds = 0.0f;   // clamped: no gradient
    const float dr = ds * sh.scale;
    // dQ_q = Σ_i dr_i K[key_i];  dK[key_i] += dr_i q;  dV[key_i] += w_i dO_q
    for (int t = lane; t < d; t += 32) {
        float acc = 0.0f;
        const float qt = to_f(Q[row * d + t]), gt = to_f(dO[row * d + t]);
        for (int j = 0; j < k; ++j) {
            const int kj = __shfl_sync(0xffffffffu, key, j);
            const float drj = __shfl_sync(0xffffffffu, dr, j);
            const float wjj = __shfl_sync(0xffffffffu, wj, j);
            if (kj < 0) continue;
            const size_t krow = (bh * sh.NK + kj) * d + t;
            acc = fmaf(drj, to_f(K[krow]), acc);
            if (drj != 0.0f) atomicAdd(dK32 + krow, drj * qt);
            atomicAdd(dV32 + krow, wjj * gt);
        }
        dQ[row * d + t] = from_f<TO>(isfinite(acc) ? acc : 0.0f);
    }
}

template <typename TO>
__global__ void convert_kernel(const float* __restrict__ a, TO* __restrict__ out, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float v = a[i];
        out[i] = from_f<TO>(isfinite(v) ? v : 0.0f);
    }
}

#define ASA_STABLE_DISPATCH(s, ...)                                                          \
    do {                                                                                     \
        if ((s).in_dtype == ASA_DTYPE_F32) {                                                 \
            using T = float;                                                                 \
            if ((s).out_dtype == ASA_DTYPE_F32) { using TO = float; __VA_ARGS__; }           \
            else { using TO = __nv_bfloat16; __VA_ARGS__; }                                  \
        } else {                                                                             \
            using T = __nv_bfloat16;                                                         \
            if ((s).out_dtype == ASA_DTYPE_F32) { using TO = float; __VA_ARGS__; }           \
            else { using TO = __nv_bfloat16; __VA_ARGS__; }                                  \
        }                                                                                    \
    } while (0)

}  // namespace

cudaError_t stable_forward(const Shape& s, float alpha, const void* V, const float* topv,
                           const int32_t* topi, void* O, float* tau, float* weights,
                           float* tau_coef, cudaStream_t st) {
    const size_t rows = (size_t)s.BH * s.NQ;
    if (!rows) return cudaSuccess;
    const unsigned grid = (unsigned)((rows + STABLE_WARPS - 1) / STABLE_WARPS);
    const float a = stable_alpha(alpha);
    ASA_STABLE_DISPATCH(s, {
        stable_fwd_kernel<T, TO><<<grid, 32 * STABLE_WARPS, 0, st>>>(s, a, (const T*)V, topv, topi, (TO*)O, tau,
                                                                     weights, tau_coef);
        note_launch();
        return cudaGetLastError();
    });
    return cudaErrorInvalidValue;
}

cudaError_t stable_backward(const Shape& s, float alpha, const void* Q, const void* K,
                            const void* V, const void* dO, const float* topv,
                            const int32_t* topi, const float* weights, const float* tau,
                            const float* tau_coef, void* dQ, float* dK32, float* dV32,
                            void* dK, void* dV, cudaStream_t st) {
    const size_t kn = (size_t)s.BH * s.NK * s.d;
    cudaError_t e = cudaMemsetAsync(dK32, 0, kn * 4, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(dV32, 0, kn * 4, st);
    if (e != cudaSuccess) return e;
    const size_t rows = (size_t)s.BH * s.NQ;
    const float a = stable_alpha(alpha);
    ASA_STABLE_DISPATCH(s, {
        if (rows) {
            const unsigned grid = (unsigned)((rows + STABLE_WARPS - 1) / STABLE_WARPS);
            stable_bwd_kernel<T, TO><<<grid, 32 * STABLE_WARPS, 0, st>>>(
                s, a, (const T*)Q, (const T*)K, (const T*)V, (const T*)dO, topv, topi, weights, tau, tau_coef,
                (TO*)dQ, dK32, dV32);
            note_launch();
            e = cudaGetLastError();
            if (e != cudaSuccess) return e;
        }
        if (kn) {
            const unsigned cg = (unsigned)((kn + 255) / 256 < 4096 ? (kn + 255) / 256 : 4096);
            convert_kernel<TO><<<cg, 256, 0, st>>>(dK32, (TO*)dK, kn);
            convert_kernel<TO><<<cg, 256, 0, st>>>(dV32, (TO*)dV, kn);
            note_launch(2);
            e = cudaGetLastError();
        }
        return e;
    });
    return cudaErrorInvalidValue;
}

}  // namespace asa
