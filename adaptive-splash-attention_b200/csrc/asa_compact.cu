// asa_compact.cu -- tile lists from the block mask, and the device-side
// scrub.
//
// build_lists: one CTA per (b,h) row turns M[nQB][nKB] into
//  * the CSR the reference builds (build_lookup_kernel :219-242):
//    csr_ptr[nQB+1] prefix sums of row counts, csr_idx the ascending active
//    key blocks of each query block, zero padded to nQB*nKB;
//  * its transpose (per key block, ascending active query blocks), which the
//    key-major backward walks.
// The reference runs this serially in 32 redundant threads per row; here
// each thread owns rows (then columns) and one warp scans the counts.
#include "asa_internal.h"

namespace asa {
namespace {

constexpr int LT = 256;

// Exclusive scan of cnt[0..n) into out[0..n] (out[n] = total) by one warp.
__device__ void warp_scan(const int* cnt, int32_t* out, int n) {
    const int lane = threadIdx.x & 31;
    int carry = 0;
    for (int base = 0; base < n; base += 32) {
        const int i = base + lane;
        int v = i < n ? cnt[i] : 0;
        int x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (i < n) out[i] = carry + x - v;
        carry += __shfl_sync(0xffffffffu, x, 31);
    }
    if (lane == 0) out[n] = carry;
}

__global__ void __launch_bounds__(LT)
build_lists_kernel(int nQB, int nKB, const uint8_t* __restrict__ M, int32_t* __restrict__ csr_ptr,
                   int32_t* __restrict__ csr_idx, int32_t* __restrict__ csc_ptr,
                   int32_t* __restrict__ csc_idx) {
    extern __shared__ int cnt[];   // max(nQB, nKB) + 1 counts, then the scan
    const int bh = blockIdx.x;
    const uint8_t* m = M + (size_t)bh * nQB * nKB;
    const size_t total = (size_t)nQB * nKB;
    for (int pass = 0; pass < 2; ++pass) {
        const bool rows = pass == 0;
        int32_t* ptr = rows ? csr_ptr : csc_ptr;
        int32_t* idx = rows ? csr_idx : csc_idx;
        if (ptr == nullptr) continue;
        const int n = rows ? nQB : nKB, w = rows ? nKB : nQB;
        ptr += (size_t)bh * (n + 1);
        idx += (size_t)bh * total;
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += LT) {
            int c = 0;
            for (int j = 0; j < w; ++j) c += rows ? m[(size_t)i * nKB + j] : m[(size_t)j * nKB + i];
            cnt[i] = c;
        }
        __syncthreads();
        if (threadIdx.x < 32) warp_scan(cnt, ptr, n);
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += LT) {
            int o = ptr[i];
            for (int j = 0; j < w; ++j)
                if (rows ? m[(size_t)i * nKB + j] : m[(size_t)j * nKB + i]) idx[o++] = j;
        }
        const int used = ptr[n];
        for (size_t x = used + threadIdx.x; x < total; x += LT) idx[x] = 0;
    }
}

template <typename T>
__global__ void scrub_detect(const T* __restrict__ x, size_t n, int* flag) {
    int inf = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        inf |= isinf(to_f(x[i])) ? 1 : 0;
    if (__syncthreads_or(inf) && threadIdx.x == 0) atomicOr(flag, 1);
}

template <typename T>
__global__ void scrub_apply(T* __restrict__ x, size_t n, const int* flag) {
    const bool clamp = *flag != 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float v = to_f(x[i]);
        if (isnan(v)) v = 0.0f;                               // :601, :687
        if (clamp) v = fminf(fmaxf(v, -100.0f), 100.0f);      // :605, :691
        x[i] = from_f<T>(v);
    }
}

}  // namespace

cudaError_t build_lists(const Shape& s, const uint8_t* M, int32_t* csr_ptr, int32_t* csr_idx,
                        int32_t* csc_ptr, int32_t* csc_idx, cudaStream_t st) {
    const int n = (s.nQB > s.nKB ? s.nQB : s.nKB) + 1;
    const size_t smem = sizeof(int) * (size_t)n;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(build_lists_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    build_lists_kernel<<<s.BH, LT, smem, st>>>(s.nQB, s.nKB, M, csr_ptr, csr_idx, csc_ptr, csc_idx);
    note_launch();
    return cudaGetLastError();
}

cudaError_t scrub(int dtype, void* x, size_t n, int* flag, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(int), st);
    if (e != cudaSuccess) return e;
    const int blocks = 148 * 4;
    if (dtype == ASA_DTYPE_F32) {
        scrub_detect<float><<<blocks, 256, 0, st>>>((const float*)x, n, flag);
        scrub_apply<float><<<blocks, 256, 0, st>>>((float*)x, n, flag);
    } else {
        scrub_detect<__nv_bfloat16><<<blocks, 256, 0, st>>>((const __nv_bfloat16*)x, n, flag);
        scrub_apply<__nv_bfloat16><<<blocks, 256, 0, st>>>((__nv_bfloat16*)x, n, flag);
    }
    note_launch(2);
    return cudaGetLastError();
}

}  // namespace asa
