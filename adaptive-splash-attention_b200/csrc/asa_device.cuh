// asa_device.cuh -- device helpers shared by the SIMT and tcgen05 kernels:
// element loads, the top-k list, the reference τ solve and the entmax
// transform.
//
// Floating-point rule: the τ solve and the SIMT paths reproduce the
// reference's arithmetic (source/adasplashattention.cu) step for step.  The
// intrinsics __fmul_rn / __fadd_rn / __fmaf_rn pin every rounding so the
// compiler cannot contract a product into a neighbouring add differently
// from the fused steps written out here.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define ASA_EPS 1e-8f        // reference EPS (:21)
#define ASA_HALLEY_ITERS 5   // reference MAX_HALLEY_ITERS (:22)
#define ASA_SENTINEL (-1e6f) // reference top-k seed value (:170)

namespace asa {

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
    return __float2bfloat16_rn(x);
}

__device__ __forceinline__ bool finite(float x) { return isfinite(x); }

// Score as the reference forms it: raw dot · sm_scale, clamped to [-10, 10]
// (:195-197, :306-309, :415-418).
__device__ __forceinline__ float clamp_score(float raw, float sm_scale) {
    float s = __fmul_rn(raw, sm_scale);
    s = fmaxf(s, -10.0f);
    return fminf(s, 10.0f);
}

// x^e for the exponents the reference's powf calls take.  Integer exponents
// in {-1, 0, 1, 2, 3, 4} (every α with 1/(α-1) integral: 2, 1.5, 1.25, ...)
// are computed exactly rounded: x*x is correctly rounded, x^3 and x^4 go
// through double (x^2 is exact there) and round once more to float.  Any
// other exponent calls powf.
struct PowSpec {
    int kind;  // 0 powf, 1 x, 2 x^2, 3 x^3, 4 x^4, 5 one, 6 1/x
    float e;
};

__host__ __device__ inline PowSpec make_pow(float e) {
    PowSpec s;
    s.e = e;
    s.kind = 0;
    if (e == 1.0f) s.kind = 1;
    else if (e == 2.0f) s.kind = 2;
    else if (e == 3.0f) s.kind = 3;
    else if (e == 4.0f) s.kind = 4;
    else if (e == 0.0f) s.kind = 5;
    else if (e == -1.0f) s.kind = 6;
    return s;
}

__device__ __forceinline__ float pow_exact(float x, PowSpec s) {
    switch (s.kind) {
        case 1: return x;
        case 2: return __fmul_rn(x, x);
        case 3: { double x2 = (double)x * (double)x; return (float)(x2 * (double)x); }
        case 4: { double x2 = (double)x * (double)x; return (float)(x2 * x2); }
        case 5: return 1.0f;
        case 6: return __fdiv_rn(1.0f, x);
        default: return powf(x, s.e);
    }
}

// pow_exact with the exponent class fixed at compile time (same arithmetic
// per kind; KIND 0 classifies the runtime exponent as pow_exact does).
template <int KIND>
__device__ __forceinline__ float pow_exact_k(float x, float e) {
    if constexpr (KIND == 1) return x;
    else if constexpr (KIND == 2) return __fmul_rn(x, x);
    else if constexpr (KIND == 3) { double x2 = (double)x * (double)x; return (float)(x2 * (double)x); }
    else if constexpr (KIND == 4) { double x2 = (double)x * (double)x; return (float)(x2 * x2); }
    else if constexpr (KIND == 5) return 1.0f;
    else if constexpr (KIND == 6) return __fdiv_rn(1.0f, x);
    else return pow_exact(x, make_pow(e));
}

// Reference entmax p for one score (:311-316): u = (α-1)s - τ;
// p = u > 0 ? max(u, EPS)^{1/(α-1)} : 0; non-finite -> 0.
__device__ __forceinline__ float entmax_p(float s, float am1, float tau, PowSpec pinv, float* u_out) {
    float u = __fmaf_rn(am1, s, -tau);
    float p = (u > 0.0f) ? pow_exact(fmaxf(u, ASA_EPS), pinv) : 0.0f;
    if (!isfinite(p)) p = 0.0f;
    *u_out = u;
    return p;
}

// Top-k list of the reference (:35-49, seeded :166-172) for a runtime k <= KM.
// Slots [0, KM-k) hold +inf "phantom" entries that no score can displace, so
// the live list is slots [KM-k, KM) and insertion is a fixed, fully unrolled
// compare-and-shift network: entry j takes the new value when it is the
// first slot the value beats, the entry above it when the value also beats
// that one.  Strict '>' keeps the earlier key on ties, as the reference does.
template <int KM>
struct TopK {
    float v[KM];
    int i[KM];

    __device__ __forceinline__ void init(int k) {
#pragma unroll
        for (int j = 0; j < KM; ++j) {
            bool live = j >= KM - k;
            v[j] = live ? ASA_SENTINEL : __int_as_float(0x7f800000);
            i[j] = live ? -1 : -2;
        }
    }
    __device__ __forceinline__ float threshold() const { return v[KM - 1]; }
    // Insert under the total order (value desc, key index asc): used to merge
    // two partial lists of disjoint key sets; the result is the first k of
    // that order, exactly what sequential strict-'>' insertion in key order
    // keeps.
    __device__ __forceinline__ void insert_lex(float s, int idx) {
#pragma unroll
        for (int j = KM - 1; j >= 0; --j) {
            const bool gt = s > v[j] || (s == v[j] && idx < i[j]);
            const bool gt_up = (j > 0) ? (s > v[j - 1] || (s == v[j - 1] && idx < i[j - 1])) : false;
            if (gt) {
                v[j] = gt_up ? v[j - 1] : s;
                i[j] = gt_up ? i[j - 1] : idx;
            }
        }
    }
    __device__ __forceinline__ void insert(float s, int idx) {
#pragma unroll
        for (int j = KM - 1; j >= 0; --j) {
            bool gt = s > v[j];
            bool gt_up = (j > 0) ? (s > v[j - 1]) : false;
            if (gt) {
                v[j] = gt_up ? v[j - 1] : s;
                i[j] = gt_up ? i[j - 1] : idx;
            }
        }
    }
};

// Reference τ solve (entmax_threshold with full=true, :51-148) over the live
// slots [KM-k, KM) of a TopK list.  At most five Halley steps with the
// reference's bracket, early exit |f| < 1e-4, bisection fallback, per-step
// clamp and second-derivative coefficient inv·(inv+1-α) (:85).
template <int KM, int K1, int K2, int K3>
__device__ __forceinline__ float ref_tau_k(const float (&s)[KM], int k, float alpha_in) {
    const float alpha = fmaxf(1.05f, fminf(alpha_in, 3.0f));
    const float am1 = __fadd_rn(alpha, -1.0f);
    const float inv = __fdiv_rn(1.0f, am1);
    const float e2 = __fmul_rn(__fadd_rn(2.0f, -alpha), inv);
    const float e3 = __fmul_rn(__fadd_rn(3.0f, -__fmul_rn(2.0f, alpha)), inv);
    const float c2 = __fmul_rn(inv, __fadd_rn(__fadd_rn(inv, 1.0f), -alpha));
    const int first = KM - k;
    float s_max = s[KM - 1];
#pragma unroll
    for (int j = 0; j < KM; ++j)
        if (j == first) s_max = s[j];   // unrolled select: no dynamically indexed (local) array
    const float s_min = s[KM - 1];
    float lo = __fmaf_rn(am1, s_min, -2.0f);
    float hi = __fmaf_rn(am1, s_max, 2.0f);
    float tau = __fmul_rn(0.5f, __fadd_rn(lo, hi));
    for (int it = 0; it < ASA_HALLEY_ITERS; ++it) {
        float f = -1.0f, fp = 0.0f, fpp = 0.0f;
        bool alive = true;
#pragma unroll
        for (int j = 0; j < KM; ++j) {
            if (j < first) continue;
            float u = __fmaf_rn(am1, s[j], -tau);
            alive = alive && (u > 0.0f);   // the reference breaks at the first u <= 0
            if (alive) {
                float uc = fmaxf(u, ASA_EPS);
                float up = pow_exact_k<K1>(uc, inv);
                if (!isfinite(up)) up = 0.0f;
                f = __fadd_rn(f, up);
                float dt = __fmul_rn(-inv, pow_exact_k<K2>(uc, e2));
                if (isfinite(dt)) fp = __fadd_rn(fp, dt);
                float st = __fmul_rn(c2, pow_exact_k<K3>(uc, e3));
                if (isfinite(st)) fpp = __fadd_rn(fpp, st);
            }
        }
        if (fabsf(f) < 1e-4f) break;
        float tn = tau;
        if (fabsf(fp) > ASA_EPS) {
            float denom = __fmaf_rn(__fmul_rn(2.0f, fp), fp, -__fmul_rn(f, fpp));
            if (fabsf(denom) > ASA_EPS)
                tn = __fadd_rn(tau, -__fdiv_rn(__fmul_rn(__fmul_rn(2.0f, f), fp), denom));
        }
        if (!(tn >= lo && tn <= hi)) tn = __fmul_rn(0.5f, __fadd_rn(lo, hi));
        f = -1.0f;
        alive = true;
#pragma unroll
        for (int j = 0; j < KM; ++j) {
            if (j < first) continue;
            float u = __fmaf_rn(am1, s[j], -tn);
            alive = alive && (u > 0.0f);
            if (alive) {
                float up = pow_exact_k<K1>(fmaxf(u, ASA_EPS), inv);
                if (isfinite(up)) f = __fadd_rn(f, up);
            }
        }
        if (f > 0.0f) lo = tn; else hi = tn;
        tau = tn;
        tau = fmaxf(tau, __fmaf_rn(s_min, am1, -10.0f));
        tau = fminf(tau, __fmaf_rn(s_max, am1, 10.0f));
    }
    return tau;
}


// Runtime dispatch over the exponent classes of α = 1.5, 2 and 1.25 (whose
// τ-solve exponents are all exact small powers); other α take the powf
// instantiation.  Compile-time classes keep the solve branch-free per
// element: a runtime switch per pow costs ~3x the whole solve.
template <int KM>
__device__ float ref_tau(const float (&s)[KM], int k, float alpha_in) {
    const float alpha = fmaxf(1.05f, fminf(alpha_in, 3.0f));
    const float am1 = __fadd_rn(alpha, -1.0f);
    const float inv = __fdiv_rn(1.0f, am1);
    const int k1 = make_pow(inv).kind;
    const int k2 = make_pow(__fmul_rn(__fadd_rn(2.0f, -alpha), inv)).kind;
    const int k3 = make_pow(__fmul_rn(__fadd_rn(3.0f, -__fmul_rn(2.0f, alpha)), inv)).kind;
    if (k1 == 2 && k2 == 1 && k3 == 5) return ref_tau_k<KM, 2, 1, 5>(s, k, alpha_in);   // α = 1.5
    if (k1 == 1 && k2 == 5 && k3 == 6) return ref_tau_k<KM, 1, 5, 6>(s, k, alpha_in);   // α = 2
    if (k1 == 4 && k2 == 3 && k3 == 2) return ref_tau_k<KM, 4, 3, 2>(s, k, alpha_in);   // α = 1.25
    return ref_tau_k<KM, 0, 0, 0>(s, k, alpha_in);
}

// Record an error code in the device error word (first error wins).  The
// word lives in the C-ABI translation unit; kernels receive its address.
__device__ __forceinline__ void raise_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

}  // namespace asa
