// asa_tc.cu -- tcgen05 / TMEM / TMA kernels for bf16 inputs, head dim 64 or
// 128, 128x128 mask tiles.
//
// Kernels (one CTA per 128-row block, warp-specialised):
//   tc_bounds    per-block min/max of the position indices (tile visibility)
//   k1_tau_mask  top-k and block mask: S = Q·K^T over every visible tile into
//                TMEM (four buffers), epilogue warps stream each score row
//                through the reference top-k (reference build_mask_kernel
//                :150-217); k1_tau_solve then solves τ per row
//   k13_fused    k1_tau_mask and k3_forward in one CTA per query block: top-k,
//                τ from the merged lists, then the forward over the block's
//                active key blocks (no tile lists read; Q loaded once)
//   k3_forward   O = Σ p v / (Σ p + EPS) over the CSR tile list: S = Q·K^T,
//                entmax p in the epilogue warps, P written back to TMEM as a
//                bf16 hi/lo pair, O += P_hi·V + P_lo·V in TMEM
//                (reference splash_forward_sparse :244-341)
//   k4_pre       D_q = O·dO per query (the acc·dO/n term of :487-491)
//   k4_dq        dQ = Σ dS·K over the CSR list (query-major)
//   k4_dkdv      dV = Σ P^T·dO/n, dK = Σ dS^T·Q over the transposed list
//                (key-major; no atomics)
//                (reference splash_backward_sparse :343-535)
//
// Warp roles: warp 0 issues the TMA loads, warp 1 owns TMEM and issues MMAs
// (lane 0), in the forward and backward warp 2 issues the second MMA stream,
// and the remaining warps are the epilogue: thread (warp%4)*32+lane owns
// TMEM lane = tile row.  The epilogue warps also apply the reference's
// tile-load zeroing to freshly loaded K/V tiles that need it.
//
// Every mbarrier wait is bounded (Shape::spins polls); when one runs out the
// kernel records ASA_ERR_DEVICE_TIMEOUT in the device error word and carries
// on without the data, so it always terminates; before exiting, its TMA and
// MMA issuers wait (with a fixed bound) for their own work still in flight.
#include "asa_internal.h"
#include "asa_sm100.cuh"
#include <climits>
#include <cstdio>
#include <cudaTypedefs.h>
#include <type_traits>

namespace asa {

struct Bounds {
    const int* qmin;   // [BH][nQB]
    const int* qmax;
    const int* kmin;   // [BH][nKB]
    const int* kmax;
};

namespace {

using namespace sm100;

constexpr int TILE = 128;
constexpr int BOX = 64;                    // bf16 elements per 128-byte swizzle row
constexpr int BOX_BYTES = TILE * 128;      // one 64-column box of 128 rows
constexpr int NEPI = 256;                  // threads that build a CTA's tile schedule (epi_bar counts them)
constexpr int EPI0 = 64;                   // τ / mask: first epilogue thread (producer and MMA warps first)
constexpr int K3_EPI0 = 96;                // forward: producer, S-issuer and P·V-issuer warps first
constexpr int DQ_NW = 4;                   // dQ: epilogue warpgroups (one 32-column chunk each)
constexpr int DQ_NE = 128 * DQ_NW;
constexpr int DQ_EPI0 = 96;                // dQ: producer, S/dP-issuer and dQ-issuer warps first
constexpr int DQ_THREADS = DQ_EPI0 + DQ_NE;
constexpr int DKV_NW = 4;                  // dK/dV: epilogue warpgroups (32 queries of a tile each)
constexpr int DKV_NE = 128 * DKV_NW;
constexpr int DKV_EPI0 = 96;               // dK/dV: producer, S/dP-issuer and dV/dK-issuer warps first
constexpr int DKV_THREADS = DKV_EPI0 + DKV_NE;


// Dynamic shared memory starts at the bottom of the CTA's window (these
// kernels declare no static __shared__ data), which is 1024-byte aligned as
// the 128-byte swizzle atoms require.  A misaligned base is reported, not
// silently mis-swizzled.
__device__ __forceinline__ uint8_t* align1024(uint8_t* p, int* err) {
    if ((smem_u32(p) & 1023u) != 0 && threadIdx.x == 0 && err) atomicCAS(err, 0, ASA_ERR_UNSUPPORTED);
    return p;
}

__device__ __forceinline__ void epi_bar() {
    asm volatile("bar.sync 1, %0;" ::"n"(NEPI) : "memory");
}

__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }

// One arrival per epilogue warp (barriers are initialised with the epilogue
// warp count): the warp's prior writes and tcgen05 fences are ordered before
// lane 0's arrive by __syncwarp.
__device__ __forceinline__ void epi_arrive(uint64_t* bar) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) sm100::mbar_arrive(bar);
}

// ---- tile classification (identical in every role) --------------------------
__device__ __forceinline__ bool vis_any(const Shape& s, const Bounds& b, int bh, int qb, int kb) {
    if (!s.causal) return true;
    return b.kmin[bh * s.nKB + kb] <= b.qmax[bh * s.nQB + qb];
}
__device__ __forceinline__ bool vis_all(const Shape& s, const Bounds& b, int bh, int qb, int kb) {
    if ((kb + 1) * TILE > s.NK) return false;
    if (!s.causal) return true;
    return b.kmax[bh * s.nKB + kb] <= b.qmin[bh * s.nQB + qb];
}
__device__ __forceinline__ bool needs_fix(const Shape& s, const Bounds& b, int bh, int qb, int kb) {
    if (!s.ref_load || !s.causal) return false;   // bounds exist only for causal shapes
    return b.kmax[bh * s.nKB + kb] > b.qmin[bh * s.nQB + qb];
}

// Block order of the one-dimensional grids over (head, row block): groups
// of kGroupHeads heads, and inside a group the heads fastest, so each group's
// heaviest blocks (causal: the last query blocks) are dispatched first while
// the K/V of only a few heads are live in L2 at a time.  Returns (head,
// block); reverse: block nb-1 is the first dispatched.
constexpr int kGroupHeads = 4;
__device__ __forceinline__ int2 grid_order(int BH, int nb, bool reverse) {
    const int L = (int)blockIdx.x;
    const int g = L / (kGroupHeads * nb);
    const int gh = min(kGroupHeads, BH - g * kGroupHeads);
    const int idx = L - g * kGroupHeads * nb;
    const int rank = idx / gh;
    return make_int2(g * kGroupHeads + idx % gh, reverse ? nb - 1 - rank : rank);
}

// ---- per-CTA tile schedule ----------------------------------------------------
// Each CTA stages its tile sequence in shared memory once, so no role chases
// a global list -> bounds dependency per tile: entry = block index (low 24
// bits) | SCHED_ALL (every pair of the tile visible) | SCHED_FIX (the
// reference's tile-load zeroing can apply).
constexpr uint32_t SCHED_IDX = (1u << 24) - 1, SCHED_ALL = 1u << 30, SCHED_FIX = 1u << 31;

__device__ __forceinline__ uint32_t sched_entry(const Shape& s, const Bounds& bd, int bh, int qb, int kb,
                                                int idx) {
    uint32_t e = (uint32_t)idx;
    if (vis_all(s, bd, bh, qb, kb) && (qb + 1) * TILE <= s.NQ) e |= SCHED_ALL;
    if (needs_fix(s, bd, bh, qb, kb)) e |= SCHED_FIX;
    return e;
}

// Schedule from a CSR (query-major: fixed qb, list of kb) or transposed
// (key-major: fixed kb, list of qb) tile list; run by the epilogue threads.
__device__ __forceinline__ void sched_from_list(uint32_t* sched, const int32_t* __restrict__ list, int T,
                                                const Shape& s, const Bounds& bd, int bh, int fixed,
                                                bool key_major, int et) {
    for (int t = et; t < T; t += NEPI) {
        const int other = list[t];
        sched[t] = key_major ? sched_entry(s, bd, bh, other, fixed, other)
                             : sched_entry(s, bd, bh, fixed, other, other);
    }
}

// Schedule of every key block with a visible pair for query block qb (the
// τ / mask pass), compacted in ascending order.  Returns the count; run by
// the 256 epilogue threads (warp_cnt: 8 ints of shared memory).
__device__ int sched_visible(uint32_t* sched, int* warp_cnt, const Shape& s, const Bounds& bd, int bh,
                             int qb, int et) {
    const int w = et >> 5, lane = et & 31;
    int total = 0;
    for (int base = 0; base < s.nKB; base += NEPI) {
        const int kb = base + et;
        const bool v = kb < s.nKB && vis_any(s, bd, bh, qb, kb);
        const uint32_t bal = __ballot_sync(0xffffffffu, v);
        if (lane == 0) warp_cnt[w] = __popc(bal);
        epi_bar();
        int before = 0, all = 0;
        for (int i = 0; i < NEPI / 32; ++i) {
            before += i < w ? warp_cnt[i] : 0;
            all += warp_cnt[i];
        }
        if (v) sched[total + before + __popc(bal & ((1u << lane) - 1))] = sched_entry(s, bd, bh, qb, kb, kb);
        total += all;
        epi_bar();
    }
    return total;
}

// ---- the reference's tile-load zeroing on a swizzled 128-row tile ------------
// Element (row r, dim t) of key kb*128+r is zeroed for query block qb when the
// reference thread that stages it (query qb*128 + ((r*d + t) % 128)) cannot
// see the key.  qidx_blk holds that block's 128 positions (INT_MAX past NQ,
// which keeps the element, see ref_keep).  Executed by one full warp.
template <int D>
__device__ __forceinline__ uint4* fix_chunk(uint8_t* tile, int r, int t0) {
    const int phys = ((t0 % BOX) / 8) ^ (r & 7);
    return reinterpret_cast<uint4*>(tile + (t0 / BOX) * BOX_BYTES + r * 128 + phys * 16);
}

// Zero the elements of one 16-byte chunk whose bit in `keep` is clear.
__device__ __forceinline__ void fix_apply(uint4* p, uint32_t keep) {
    uint4 v = *p;
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 8; ++e)
        if (!((keep >> e) & 1u)) w[e >> 1] &= (e & 1) ? 0x0000ffffu : 0xffff0000u;
    *p = make_uint4(w[0], w[1], w[2], w[3]);
}

// Rows row0 + lane + 32*rr (rr < NR) of the tile; fix_tile: all 128 rows
// by one warp.
template <int D, int NR = TILE / 32>
__device__ void fix_tile(uint8_t* tile, const int* qidx_blk, int qmin_blk,
                         const int32_t* __restrict__ Kidx_bh, int kb, int NK, int lane, int row0 = 0) {
    static_assert(D == 64 || D == 128, "staging windows assume D in {64, 128}");
    int kp[NR];
#pragma unroll
    for (int rr = 0; rr < NR; ++rr) {     // independent loads: one latency for all rows
        const int kn = kb * TILE + row0 + lane + 32 * rr;
        kp[rr] = kn < NK ? __ldg(Kidx_bh + kn) : INT_MIN;
    }
    // Row r's staging queries for dims 0..D-1 are the contiguous window
    // [(r*D) % 128, (r*D) % 128 + D).  When the block's positions are
    // nondecreasing (the usual arange case) the zeroed dims of a row are a
    // prefix [0, n) with n = #{t : qidx[window + t] < kpos}: a branch-free
    // binary search, then whole-chunk zero stores.
    const int4 q4 = reinterpret_cast<const int4*>(qidx_blk)[lane];
    const int qnext = lane < 31 ? qidx_blk[4 * lane + 4] : INT_MAX;
    const bool mono = __all_sync(0xffffffffu, q4.x <= q4.y && q4.y <= q4.z && q4.z <= q4.w && q4.w <= qnext);
#pragma unroll
    for (int rr = 0; rr < NR; ++rr) {
        const int r = row0 + lane + 32 * rr;
        const int kpos = kp[rr];
        if (kpos <= qmin_blk) continue;          // every staging query sees the key
        const int base = (r * D) & (TILE - 1);
        if (mono) {
            int n = 0;
#pragma unroll
            for (int step = D / 2; step >= 1; step >>= 1)
                if (qidx_blk[base + n + step - 1] < kpos) n += step;
#pragma unroll
            for (int ch = 0; ch < D / 8; ++ch) {
                if ((ch + 1) * 8 <= n) *fix_chunk<D>(tile, r, ch * 8) = make_uint4(0u, 0u, 0u, 0u);
                else if (ch * 8 < n) fix_apply(fix_chunk<D>(tile, r, ch * 8), 0xffu << (n - ch * 8));
            }
        } else {
#pragma unroll 2
            for (int ch = 0; ch < D / 8; ++ch) {
                // the 8 staging queries of this 16-byte chunk are consecutive
                const int4* qp = reinterpret_cast<const int4*>(qidx_blk + base + ch * 8);
                const int4 qa = qp[0], qc = qp[1];
                const uint32_t keep = (kpos <= qa.x ? 1u : 0u) | (kpos <= qa.y ? 2u : 0u) |
                                      (kpos <= qa.z ? 4u : 0u) | (kpos <= qa.w ? 8u : 0u) |
                                      (kpos <= qc.x ? 16u : 0u) | (kpos <= qc.y ? 32u : 0u) |
                                      (kpos <= qc.z ? 64u : 0u) | (kpos <= qc.w ? 128u : 0u);
                if (keep != 0xffu) fix_apply(fix_chunk<D>(tile, r, ch * 8), keep);
            }
        }
    }
}

// ---- descriptors ---------------------------------------------------------------
// K-major operand tile (128 rows, D columns as D/64 boxes of 16 KB): k-step kk
// covers columns [16kk, 16kk+16).
__device__ __forceinline__ uint64_t kdesc(const uint8_t* tile, int kk) {
    return sdesc(smem_u32(tile + (kk >> 2) * BOX_BYTES + (kk & 3) * 32), 16, 1024);
}
// MN-major operand tile (128 K-rows of 128 bytes per 64-wide M/N box): k-step
// kk covers rows [16kk, 16kk+16); boxes are BOX_BYTES apart along M/N.
__device__ __forceinline__ uint64_t mndesc(const uint8_t* tile, int kk) {
    return sdesc(smem_u32(tile + kk * 16 * 128), BOX_BYTES, 1024);
}
// The same descriptors from a base descriptor of the tile: k-steps only move
// the 14-bit start-address field (shared addresses stay below 2^18 bytes).
__device__ __forceinline__ uint64_t kdesc_step(uint64_t base, int kk) {
    return base + (uint64_t)((((kk >> 2) * BOX_BYTES) + (kk & 3) * 32) >> 4);
}
__device__ __forceinline__ uint64_t mndesc_step(uint64_t base, int kk) {
    return base + (uint64_t)((kk * 16 * 128) >> 4);
}

// Store 32 consecutive columns [32c, 32c+32) of row `row` of a 128x128 bf16
// K-major swizzled tile from packed pairs (pk[m] = cols 2m, 2m+1).
__device__ __forceinline__ void store_row_chunk(uint8_t* tile, int row, int c, const uint32_t (&pk)[16]) {
    const int box = c >> 1;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int ch = (c & 1) * 4 + i;
        const int phys = ch ^ (row & 7);
        uint4* p = reinterpret_cast<uint4*>(tile + box * BOX_BYTES + row * 128 + phys * 16);
        *p = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
    }
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Packed (two-lane fp32) entmax weights for exponent classes 1, 2 and 4:
// u = clamp(c1·raw - τ) with c1 = (α-1)·sm_scale, upper bound (α-1)·10 - τ
// and lower bound 0 (callers take this path only when (α-1)·(-10) - τ <= 0,
// so the score clamp at -10 can only meet u <= 0, where p = 0).  The EPS
// floor of the reference changes p only below 1e-16 (exponent 2) and is
// dropped.  p pairs are split into bf16 hi (rounded) and lo (remainder)
// halves packed two per 32-bit word; the row sum gathers in two lanes.
template <int PK>
__device__ __forceinline__ float2 entmax_pair(uint32_t r0, uint32_t r1, float2 c1, float2 mtau, float uhi) {
    float2 u = __ffma2_rn(make_float2(__uint_as_float(r0), __uint_as_float(r1)), c1, mtau);
    u.x = fmaxf(fminf(u.x, uhi), 0.0f);
    u.y = fmaxf(fminf(u.y, uhi), 0.0f);
    if constexpr (PK == 1) return u;
    else if constexpr (PK == 2) return __fmul2_rn(u, u);
    else { const float2 q = __fmul2_rn(u, u); return __fmul2_rn(q, q); }
}
__device__ __forceinline__ void split_pair(float2 p, uint32_t& hi, uint32_t& lo) {
    hi = pack_bf16(p.x, p.y);
    const float2 hf = make_float2(__uint_as_float(hi << 16), __uint_as_float(hi & 0xffff0000u));
    const float2 l = __ffma2_rn(hf, make_float2(-1.0f, -1.0f), p);
    lo = pack_bf16(l.x, l.y);
}

// hi/lo split of 32 values: hi = bf16(x), lo = bf16(x - hi).  With split=false
// only hi is produced (lo left untouched).
__device__ __forceinline__ void split_pack(const float (&x)[32], uint32_t (&hi)[16], uint32_t (&lo)[16]) {
#pragma unroll
    for (int m = 0; m < 16; ++m) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * m], x[2 * m + 1]);
        hi[m] = *reinterpret_cast<const uint32_t*>(&h);
        const float2 hf = __bfloat1622float2(h);
        lo[m] = pack_bf16(x[2 * m] - hf.x, x[2 * m + 1] - hf.y);
    }
}


// x^e with the exponent class fixed at compile time (PK = PowSpec kind:
// 1 x, 2 x^2, 3 x^3, 4 x^4, 5 one, 0 powf with runtime e).
template <int PK>
__device__ __forceinline__ float powk(float x, float e) {
    if constexpr (PK == 1) return x;
    else if constexpr (PK == 2) return x * x;
    else if constexpr (PK == 3) return x * x * x;
    else if constexpr (PK == 4) { const float y = x * x; return y * y; }
    else if constexpr (PK == 5) return 1.0f;
    else return powf(x, e);
}

// Maximum of three floats in one instruction (PTX max.f32 with three
// operands, sm_100); NaN operands are ignored as fmaxf ignores them.
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
// Largest of 32 raw scores (as bit patterns), 16 three-input maxima; m
// receives the maxima of the groups {3g, 3g+1, 3g+2} (g < 10) and {30, 31}.
__device__ __forceinline__ float chunk_max(const uint32_t (&r)[32], float (&m)[11]) {
#pragma unroll
    for (int g = 0; g < 10; ++g)
        m[g] = max3f(__uint_as_float(r[3 * g]), __uint_as_float(r[3 * g + 1]), __uint_as_float(r[3 * g + 2]));
    m[10] = fmaxf(__uint_as_float(r[30]), __uint_as_float(r[31]));
    const float a = max3f(m[0], m[1], m[2]), b = max3f(m[3], m[4], m[5]), c = max3f(m[6], m[7], m[8]);
    return fmaxf(max3f(a, b, c), fmaxf(m[9], m[10]));
}

// x^e for two values at once, exponent class PK in {1, 2, 3, 4, 5} (5: x^0).
template <int PK>
__device__ __forceinline__ float2 powk2(float2 x) {
    if constexpr (PK == 1) return x;
    else if constexpr (PK == 2) return __fmul2_rn(x, x);
    else if constexpr (PK == 3) return __fmul2_rn(__fmul2_rn(x, x), x);
    else if constexpr (PK == 4) { const float2 y = __fmul2_rn(x, x); return __fmul2_rn(y, y); }
    else return make_float2(1.0f, 1.0f);
}

// Sums over one 32-key chunk for the exact-τ solve: F += Σ u_+^{1/(α-1)},
// W += Σ u_+^{(2-α)/(α-1)} with u = (α-1)·clamp(raw·scale) - τ over the
// visible keys (bit i of vis), and hit |= any visible u > 0 at τ = tlo.
// Packed two-lane arithmetic for the exponent classes of α = 1.25, 1.5, 2
// (scale > 0); powf otherwise.
template <int PINV, int PE2>
__device__ __forceinline__ void exact_sums(const uint32_t (&r)[32], uint32_t vis, const Shape& s, float tq,
                                           float tlo, bool last, float& F, float& W, bool& hit) {
    constexpr bool kPacked = (PINV == 1 || PINV == 2 || PINV == 4) && (PE2 == 1 || PE2 == 3 || PE2 == 5);
    if (kPacked && s.scale > 0.0f) {
        const float c = __fmul_rn(s.am1, s.scale);
        const float2 c1 = make_float2(c, c), mt = make_float2(-tq, -tq), ml = make_float2(-tlo, -tlo);
        // the score clamp, as bounds on u
        const float uhi = __fmaf_rn(s.am1, 10.0f, -tq), ulo = __fmaf_rn(s.am1, -10.0f, -tq);
        const float lhi = __fmaf_rn(s.am1, 10.0f, -tlo), llo = __fmaf_rn(s.am1, -10.0f, -tlo);
        float2 f2 = make_float2(0.0f, 0.0f), w2 = make_float2(0.0f, 0.0f);
        bool h = false;
#pragma unroll
        for (int m = 0; m < 16; ++m) {
            const float2 x = make_float2(__uint_as_float(r[2 * m]), __uint_as_float(r[2 * m + 1]));
            const bool v0 = (vis >> (2 * m)) & 1u, v1 = (vis >> (2 * m + 1)) & 1u;
            float2 u = __ffma2_rn(x, c1, mt);
            u.x = v0 ? fminf(fmaxf(u.x, ulo), uhi) : 0.0f;
            u.y = v1 ? fminf(fmaxf(u.y, ulo), uhi) : 0.0f;
            const float2 up = make_float2(fmaxf(u.x, 0.0f), fmaxf(u.y, 0.0f));
            f2 = __fadd2_rn(f2, powk2<PINV>(up));
            if constexpr (PE2 == 5) w2 = __fadd2_rn(w2, make_float2(u.x > 0.0f ? 1.0f : 0.0f, u.y > 0.0f ? 1.0f : 0.0f));
            else w2 = __fadd2_rn(w2, powk2<PE2>(up));
            if (last) {
                const float2 ul = __ffma2_rn(x, c1, ml);
                h |= (v0 && fminf(fmaxf(ul.x, llo), lhi) > 0.0f) || (v1 && fminf(fmaxf(ul.y, llo), lhi) > 0.0f);
            }
        }
        F += f2.x + f2.y;
        W += w2.x + w2.y;
        hit |= h;
        return;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        if (!((vis >> i) & 1u)) continue;
        const float sc = clamp_score(__uint_as_float(r[i]), s.scale);
        const float u = __fmaf_rn(s.am1, sc, -tq);
        if (u > 0.0f) {
            const float p = powk<PINV>(u, s.pinv.e), w = powk<PE2>(u, s.pe2.e);
            if (isfinite(p)) F += p;
            if (isfinite(w)) W += w;
        }
        if (last) hit |= __fmaf_rn(s.am1, sc, -tlo) > 0.0f;
    }
}

// Entmax weight of one score (reference :311-316) for a known exponent class.
template <int PK>
__device__ __forceinline__ float entmax_pk(float u, float e) {
    float p = u > 0.0f ? powk<PK>(fmaxf(u, ASA_EPS), e) : 0.0f;
    if constexpr (PK == 0 || PK == 3 || PK == 4) p = isfinite(p) ? p : 0.0f;
    return p;
}

// Score gradient (reference :481-507): g = u^{(2-α)/(α-1)} · (dP - D) / n
// for u > EPS, else 0; non-finite -> 0.
template <int PK>
__device__ __forceinline__ float grad_pk(float u, float e, float dP, float Dq, float invN) {
    if (!(u > ASA_EPS)) return 0.0f;
    const float g = powk<PK>(fmaxf(u, ASA_EPS), e) * (dP - Dq) * invN;
    return isfinite(g) ? g : 0.0f;
}

// Visibility of keys kn0 .. kn0+31 to a query at position qpos, bit i for
// key kn0+i: the key exists (< NK) and, when causal, K_idx <= qpos.
// L1-cached position loads; only partially visible tiles need them.
__device__ __forceinline__ uint32_t vis_mask32(const int32_t* __restrict__ Kidx_bh, int kn0, int NK,
                                               int causal, int qpos) {
    const int nv = NK - kn0;
    const uint32_t exist = nv >= 32 ? 0xffffffffu : (nv <= 0 ? 0u : ((1u << nv) - 1u));
    if (!causal) return exist;
    uint32_t vis = 0;
    if (nv >= 32 && ((reinterpret_cast<uintptr_t>(Kidx_bh + kn0) & 15) == 0)) {
        const int4* p = reinterpret_cast<const int4*>(Kidx_bh + kn0);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int4 v = __ldg(p + i);
            vis |= (v.x <= qpos ? 1u : 0u) << (4 * i);
            vis |= (v.y <= qpos ? 1u : 0u) << (4 * i + 1);
            vis |= (v.z <= qpos ? 1u : 0u) << (4 * i + 2);
            vis |= (v.w <= qpos ? 1u : 0u) << (4 * i + 3);
        }
        return vis;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i)
        if (i < nv && __ldg(Kidx_bh + kn0 + i) <= qpos) vis |= 1u << i;
    return vis;
}

// Shared-memory float4 loads / stores that other threads' writes may change
// between calls (the compiler must not cache or merge them).
__device__ __forceinline__ float4 ld_volatile_f4(const float* p) {
    float4 v;
    asm volatile("ld.volatile.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(smem_u32(p)) : "memory");
    return v;
}
__device__ __forceinline__ void st_volatile_f4(float* p, float4 v) {
    asm volatile("st.volatile.shared.v4.f32 [%0], {%1, %2, %3, %4};"
                 :: "r"(smem_u32(p)), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w) : "memory");
}

__device__ __forceinline__ uint32_t tmem_lane_base(uint32_t tbase, int warp) {
    return tbase + ((uint32_t)((warp & 3) * 32) << 16);
}

// ===========================================================================
// tc_bounds: per query block min/max of Q_idx, per key block min/max of K_idx
// ===========================================================================
__global__ void tc_bounds_kernel(Shape s, const int32_t* __restrict__ Qidx,
                                 const int32_t* __restrict__ Kidx, int* qmin, int* qmax, int* kmin,
                                 int* kmax) {
    const int bh = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nwarps = blockDim.x >> 5;
    const int total = s.nQB + s.nKB;
    for (int blk = blockIdx.x * nwarps + warp; blk < total; blk += gridDim.x * nwarps) {
        const bool isq = blk < s.nQB;
        const int b = isq ? blk : blk - s.nQB;
        const int N = isq ? s.NQ : s.NK;
        const int32_t* idx = (isq ? Qidx + (size_t)bh * s.NQ : Kidx + (size_t)bh * s.NK);
        int mn = INT_MAX, mx = INT_MIN;
        for (int i = lane; i < TILE; i += 32) {
            const int n = b * TILE + i;
            if (n < N) {
                const int v = idx[n];
                mn = min(mn, v);
                mx = max(mx, v);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
            mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        }
        if (lane == 0) {
            if (isq) { qmin[bh * s.nQB + b] = mn; qmax[bh * s.nQB + b] = mx; }
            else { kmin[bh * s.nKB + b] = mn; kmax[bh * s.nKB + b] = mx; }
        }
    }
}

// ===========================================================================
// K1: τ and block mask
// ===========================================================================
// 64-bit key ordered like (value desc, key index asc) as unsigned integers:
// high word = the float's bits mapped to an increasing unsigned order, low
// word = the complement of key + 2 (keys >= -2: -2 phantom, -1 seed).
__device__ __forceinline__ unsigned long long order_key(float v, int key) {
    const uint32_t b = __float_as_uint(v);
    const uint32_t hi = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)hi << 32) | (uint32_t)(0xffffffffu - (uint32_t)(key + 2));
}

__device__ __forceinline__ float order_value(unsigned long long e) {
    const uint32_t hi = (uint32_t)(e >> 32);
    return __uint_as_float((hi & 0x80000000u) ? (hi & 0x7fffffffu) : ~hi);
}
__device__ __forceinline__ int order_index(unsigned long long e) {
    return (int)(0xffffffffu - (uint32_t)e) - 2;
}

// τ from each row's top-k scores (k1_tau_mask writes them in order, [rows][k]):
// one thread per row, so the five-step solve runs at full occupancy instead
// of in the mask kernel's tail.
template <int KM>
__global__ void __launch_bounds__(128)
k1_tau_solve(const float* __restrict__ topv, float* __restrict__ tau, size_t rows, int k, float alpha) {
    const size_t r = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    float v[KM];
#pragma unroll
    for (int i = 0; i < KM; ++i) {
        const int j = i - (KM - k);
        v[i] = j >= 0 ? topv[r * k + j] : __int_as_float(0x7f800000);
    }
    tau[r] = ref_tau<KM>(v, k, alpha);
}

// One pass over the row's visible tiles in ascending key-block order.  NW
// epilogue warpgroups split every tile by columns (warpgroup h owns keys
// [128h/NW, 128(h+1)/NW)) and keep one partial top-k list per row; the lists
// are merged pairwise under (score desc, key asc) -- the order sequential
// insertion produces.
//
// Filter.  A score can only enter the row's final list if it is >= lim, the
// largest of the partial lists' k-th values (each is a lower bound of the
// row's k-th largest; the lists publish them in shared memory after every
// tile).  lim is turned into a raw-dot bound rlo once per chunk
// (clamp(x·scale) is monotone for scale > 0; rlo sits a relative 2^-20 below
// lim/scale, so rounding can only let extra scores through), and rlo - x is
// formed with packed fp32x2 FMAs whose sign bits are funnel-shifted into a
// 32-bit candidate mask.  Candidates are read back from a per-thread
// shared-memory copy of the chunk, re-scored exactly and inserted with the
// reference's strict '>' rule, so the lists are those full insertion gives.
// On the first tile, before any list holds k scores, lim is seeded with the
// smallest of KM group maxima of the chunk (KM distinct scores of this row).
//
// The phase is written as role functions over a shared-memory view so the
// stand-alone mask kernel and the fused forward run the same code.
constexpr int MASK_S = 3;    // K stages
constexpr int MASK_NB = 4;   // S buffers in TMEM (128 columns each)

struct MaskPhase {
    uint8_t* sQ;
    uint8_t* sK;              // MASK_S stages
    float4* cbuf;             // [NE][CP][8] chunk copies
    float* thr_s;             // [NW][128] float4: published bounds (b0, b1, b2, unused)
    float* seed_s;            // [NW][128] seed bounds
    uint64_t* q_full;
    uint64_t* k_full;         // [MASK_S]
    uint64_t* k_empty;        // [MASK_S]
    uint64_t* s_full;         // [MASK_NB]
    uint64_t* s_free;         // [MASK_NB]
    uint64_t* fixed;          // K of a tile-load-zeroing tile fixed
    uint64_t* drain;          // exit-time MMA drain (after a timed-out wait)
    const int* qidx_blk;      // [128] positions of the block's queries
    const uint32_t* sched;    // [T] visible key blocks
    uint8_t* flags;           // [nKB] key blocks holding a row's top-k key
    int T;
};

// Shared memory the phase needs beyond Q and the K stages.
template <int D, int NW>
constexpr size_t mask_extra_bytes() {
    return (size_t)128 * NW * (4 / NW) * 8 * 16 + (size_t)4 * NW * TILE * 4 + (size_t)NW * TILE * 4;
}

template <int NB_>
__device__ __forceinline__ void mask_init_barriers(const MaskPhase& m, int ne) {
    mbar_init(m.q_full, 1);
    for (int i = 0; i < MASK_S; ++i) { mbar_init(&m.k_full[i], 1); mbar_init(&m.k_empty[i], 1); }
    for (int i = 0; i < NB_; ++i) { mbar_init(&m.s_full[i], 1); mbar_init(&m.s_free[i], ne / 32); }
    mbar_init(m.fixed, 4);
    mbar_init(m.drain, 1);
}

// Producer (one thread): the K tiles of the schedule through the ring.
template <int D>
__device__ void mask_produce(const MaskPhase& m, const CUtensorMap* tmK, const Shape& s, int bh, int* err) {
    constexpr int TB = D * TILE * 2;
    for (int j = 0; j < m.T; ++j) {
        const int kb = (int)(m.sched[j] & SCHED_IDX);
        const int st = j % MASK_S;
        mbar_wait(&m.k_empty[st], ((j / MASK_S) & 1) ^ 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
        mbar_expect_tx(&m.k_full[st], TB);
        for (int bx = 0; bx < D / BOX; ++bx)
            tma_load_3d(m.sK + st * TB + bx * BOX_BYTES, tmK, &m.k_full[st], bx * BOX, kb * TILE, bh);
    }
    if (error_set(err)) {   // a wait gave up: let this CTA's loads land
        mbar_drain(m.q_full, 0);
        drain_ring(m.k_full, MASK_S, m.T);
    }
}

// MMA issuer (one warp): S = Q·K^T of every scheduled tile into the TMEM
// buffers, MASK_NB in flight.
template <int D>
__device__ void mask_mma(const MaskPhase& m, const Shape& s, uint32_t tbase, int lane, int* err) {
    constexpr int TB = D * TILE * 2;
    constexpr uint32_t idesc = idesc_bf16(128, 128, 0, 0);
    mbar_wait(m.q_full, 0, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);   // issued at set-up even when T = 0
    int nfix = 0;
    for (int j = 0; j < m.T; ++j) {
        const uint32_t e = m.sched[j];
        const int st = j % MASK_S, b = j % MASK_NB;
        uint8_t* kt = m.sK + st * TB;
        mbar_wait(&m.k_full[st], (j / MASK_S) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
        if (e & SCHED_FIX)     // four epilogue warps zero K of this tile
            mbar_wait(m.fixed, (nfix++) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
        __syncwarp();
        mbar_wait(&m.s_free[b], ((j / MASK_NB) & 1) ^ 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
        tc_fence_after();
        if (lane == 0) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk)
                mma_bf16_ss(tbase + b * 128, kdesc(m.sQ, kk), kdesc(kt, kk), idesc, kk > 0);
            mma_commit(&m.s_full[b]);
            mma_commit(&m.k_empty[st]);
        }
        __syncwarp();
    }
    if (lane == 0 && error_set(err)) {   // a wait gave up: let this CTA's MMAs finish
        mma_commit(m.drain);
        mbar_drain(m.drain, 0);
    }
    __syncwarp();
}

// Epilogue thread et (row = TMEM lane, column slice h = et / 128): streams
// the row's scores of every scheduled tile through its partial top-k list.
template <int D, int KM, int NW>
__device__ void mask_epilogue(const MaskPhase& m, const Shape& s, const int32_t* __restrict__ Kidx_bh,
                              int qmin_blk, uint32_t tbase, int warp, int lane, int et, int qpos,
                              TopK<KM>& tk, int* err) {
    constexpr int NE = 128 * NW;
    constexpr int CP = 4 / NW;                // 32-column chunks per thread per tile
    constexpr int TB = D * TILE * 2;
    constexpr int GSZ = TILE / KM;            // seed group size: KM groups per tile row
    const int row = (warp & 3) * 32 + lane;
    const int h = et / TILE;
    const uint32_t tl = tmem_lane_base(tbase, warp);
    const bool scale_pos = s.scale > 0.0f;
    const float inv_scale = scale_pos ? 1.0f / s.scale : 0.0f;
    float4* my = m.cbuf + et * CP * 8;
    const int sw = lane & 7;                  // 16-byte slot swizzle: conflict-free chunk stores
    // Published bounds of the row's k-th score (each list holds distinct
    // scores): b0 = this list's k-th; b1 = its ceil(k/NW)-th (the minimum
    // over the NW lists bounds k scores); b2 = its ceil(k/2)-th (the
    // second largest over the lists bounds k scores).
    const int first = KM - s.k;
    const int i1 = first + (s.k + NW - 1) / NW - 1, i2 = first + (s.k + 1) / 2 - 1;
    tk.init(s.k);
    for (int j = 0; j < m.T; ++j) {
        const uint32_t e = m.sched[j];
        const int kb = (int)(e & SCHED_IDX);
        const int b = j % MASK_NB;
        const bool all = (e & SCHED_ALL) != 0;
        if ((e & SCHED_FIX) && et < 4 * 32) {
            // the reference's tile-load zeroing of K, 32 rows per warp
            mbar_wait(&m.k_full[j % MASK_S], (j / MASK_S) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            fix_tile<D, 1>(m.sK + (j % MASK_S) * TB, m.qidx_blk, qmin_blk, Kidx_bh, kb, s.NK, lane,
                           32 * (et >> 5));
            fence_async_smem();
            epi_arrive(m.fixed);
        }
        float lim = tk.threshold();
        {
            float m1 = __uint_as_float(0x7f800000u), x2 = neg_inf(), y2 = neg_inf();
#pragma unroll
            for (int g = 0; g < NW; ++g) {
                const float4 t = ld_volatile_f4(m.thr_s + 4 * (g * TILE + row));
                if (g != h) lim = fmaxf(lim, t.x);
                m1 = fminf(m1, t.y);
                y2 = fmaxf(y2, fminf(x2, t.z));
                x2 = fmaxf(x2, t.z);
            }
            lim = fmaxf(lim, fmaxf(m1, NW > 2 ? y2 : neg_inf()));
        }
        mbar_wait(&m.s_full[b], (j / MASK_NB) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
        tc_fence_after();
        uint32_t r2[CP][32];
#pragma unroll
        for (int cc = 0; cc < CP; ++cc) tmem_ld32(tl + b * 128 + (h * CP + cc) * 32, r2[cc]);
        tmem_ld_wait();
        tc_fence_before();
        epi_arrive(&m.s_free[b]);          // S is in registers: release the buffer
        uint32_t vis[CP];
#pragma unroll
        for (int cc = 0; cc < CP; ++cc) {
            vis[cc] = 0xffffffffu;
            if (!all) {
                vis[cc] = vis_mask32(Kidx_bh, kb * TILE + (h * CP + cc) * 32, s.NK, s.causal, qpos);
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    if (!((vis[cc] >> i) & 1u)) r2[cc][i] = 0xff800000u;   // -inf: never a candidate
            }
        }
        if (j == 0 && all && scale_pos) {
            // Seed on a fully visible first tile: the KM groups of GSZ
            // consecutive scores of the row's 128 have KM distinct
            // maxima, so the smallest bounds the row's k-th score.
            float t0 = __uint_as_float(0x7f800000u);
#pragma unroll
            for (int g = 0; g < CP * 32 / GSZ; ++g) {
                float mx = __uint_as_float(r2[(g * GSZ) / 32][(g * GSZ) % 32]);
#pragma unroll
                for (int i = 1; i < GSZ; ++i)
                    mx = fmaxf(mx, __uint_as_float(r2[(g * GSZ + i) / 32][(g * GSZ + i) % 32]));
                t0 = fminf(t0, mx);
            }
            m.seed_s[h * TILE + row] = t0;
            asm volatile("bar.sync 2, %0;" ::"n"(NE) : "memory");   // uniform: same schedule everywhere
#pragma unroll
            for (int g = 0; g < NW; ++g) t0 = fminf(t0, m.seed_s[g * TILE + row]);
            lim = fmaxf(lim, clamp_score(t0, s.scale));
        }
#pragma unroll
        for (int cc = 0; cc < CP; ++cc) {
            const int kn0 = kb * TILE + (h * CP + cc) * 32;
            const uint32_t (&r)[32] = r2[cc];
            // candidate mask: bit i set when score i may reach lim
            uint32_t cand;
            if (scale_pos && lim > -10.0f) {
                const float rlo = (lim - fmaf(fabsf(lim), 0x1p-20f, 0x1p-100f)) * inv_scale;
                const float2 lo2 = make_float2(rlo, rlo), m1 = make_float2(-1.0f, -1.0f);
                uint32_t c4[4] = {0u, 0u, 0u, 0u};
#pragma unroll
                for (int i = 3; i >= 0; --i) {
#pragma unroll
                    for (int q4 = 0; q4 < 4; ++q4) {
                        const int i0 = q4 * 8 + 2 * i;
                        const float2 dlt = __ffma2_rn(make_float2(__uint_as_float(r[i0]),
                                                                  __uint_as_float(r[i0 + 1])), m1, lo2);
                        c4[q4] = __funnelshift_l(__float_as_uint(dlt.y), c4[q4], 1);
                        c4[q4] = __funnelshift_l(__float_as_uint(dlt.x), c4[q4], 1);
                    }
                }
                cand = (c4[0] | (c4[1] << 8) | (c4[2] << 16) | (c4[3] << 24)) & vis[cc];
            } else {
                cand = vis[cc];               // no bound above the clamp floor yet: every score
            }
            if (cand) {
#pragma unroll
                for (int q8 = 0; q8 < 8; ++q8)
                    my[cc * 8 + (q8 ^ sw)] = make_float4(__uint_as_float(r[4 * q8]), __uint_as_float(r[4 * q8 + 1]),
                                                         __uint_as_float(r[4 * q8 + 2]), __uint_as_float(r[4 * q8 + 3]));
            }
            const float* myf = reinterpret_cast<const float*>(my + cc * 8);
            // the next candidate's shared-memory read is issued before the
            // current one is inserted, so its latency overlaps the insertion
            if (cand) {
                int i = __ffs(cand) - 1;
                float x = myf[(((i >> 2) ^ sw) << 2) | (i & 3)];
                for (;;) {
                    cand &= cand - 1;
                    const int ci = i;
                    const float cx = x;
                    if (cand) {
                        i = __ffs(cand) - 1;
                        x = myf[(((i >> 2) ^ sw) << 2) | (i & 3)];
                    }
                    const float v = clamp_score(cx, s.scale);
                    if (v > tk.threshold()) tk.insert(v, kn0 + ci);   // keys ascend per thread
                    if (!cand) break;
                }
            }
        }
        {
            float v1 = tk.v[KM - 1], v2 = tk.v[KM - 1];
            if (first == 0) {   // k = KM: the indices are constants
                v1 = tk.v[(KM + NW - 1) / NW - 1];
                v2 = tk.v[(KM + 1) / 2 - 1];
            } else {
#pragma unroll
                for (int i = 0; i < KM; ++i) {
                    if (i == i1) v1 = tk.v[i];
                    if (i == i2) v2 = tk.v[i];
                }
            }
            st_volatile_f4(m.thr_s + 4 * (h * TILE + row), make_float4(tk.threshold(), v1, v2, 0.0f));
        }
    }
}

// Merge: one thread per row walks the NW sorted lists (64-bit keys ordered
// like (score desc, key index asc); identical keys -- the -1e6 seeds -- go
// by list number) and emits the row's top-k in order: into topv / topi when
// given, and into mv[KM] in TopK slot layout (live slots [KM-k, KM), +inf
// before them) for a τ solve in the caller.  Marks the key blocks of the
// emitted keys in m.flags.  Run by all NE epilogue threads; `lists` is NW*KM*128
// 8-byte entries of shared memory no longer read by anyone.
template <int KM, int NW>
__device__ void mask_merge(const MaskPhase& m, const Shape& s, const TopK<KM>& tk, unsigned long long* lists,
                           int row, int h, bool qv, size_t qrow, float* __restrict__ topv,
                           int32_t* __restrict__ topi, float (&mv)[KM]) {
    constexpr int NE = 128 * NW;
    const int first = KM - s.k;
    asm volatile("bar.sync 2, %0;" ::"n"(NE) : "memory");   // K stages no longer read
#pragma unroll
    for (int i = 0; i < KM; ++i) lists[(h * KM + i) * TILE + row] = order_key(tk.v[i], tk.i[i]);
    asm volatile("bar.sync 2, %0;" ::"n"(NE) : "memory");
#pragma unroll
    for (int i = 0; i < KM; ++i) mv[i] = __int_as_float(0x7f800000);
    if (h == 0 && qv) {
        int pos[NW];
        unsigned long long cur[NW];
#pragma unroll
        for (int g = 0; g < NW; ++g) {
            pos[g] = first;
            cur[g] = lists[(g * KM + first) * TILE + row];
        }
        for (int rk = 0; rk < s.k; ++rk) {
            int bg = 0;
            unsigned long long best = cur[0];
#pragma unroll
            for (int g = 1; g < NW; ++g)
                if (cur[g] > best) { best = cur[g]; bg = g; }
            const float v = order_value(best);
            const int key = order_index(best);
            if (topv) topv[qrow * s.k + rk] = v;
            if (topi) topi[qrow * s.k + rk] = key;
#pragma unroll
            for (int i = 0; i < KM; ++i)
                if (i == first + rk) mv[i] = v;
            if (key >= 0) m.flags[key / TILE] = 1;
#pragma unroll
            for (int g = 0; g < NW; ++g)
                if (g == bg) {
                    ++pos[g];
                    cur[g] = pos[g] < KM ? lists[(g * KM + pos[g]) * TILE + row] : 0ull;
                }
        }
    }
    asm volatile("bar.sync 2, %0;" ::"n"(NE) : "memory");
}

// Stand-alone τ / mask kernel: the phase, its merge, and the mask row; τ is
// solved from the written top-k by k1_tau_solve.
template <int D, int KM, int NW>
__global__ void __launch_bounds__(64 + 128 * NW, 1)
k1_tau_mask(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK, Shape s,
            const int32_t* __restrict__ Qidx, const int32_t* __restrict__ Kidx, Bounds bd,
            float* __restrict__ topv, int32_t* __restrict__ topi, uint8_t* __restrict__ M, int* err) {
    constexpr int NE = 128 * NW;              // epilogue threads
    constexpr int TB = D * TILE * 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = align1024(smem_raw, err);
    MaskPhase m;
    m.sQ = base;
    m.sK = base + TB;
    m.cbuf = reinterpret_cast<float4*>(m.sK + MASK_S * TB);
    m.thr_s = reinterpret_cast<float*>(m.cbuf + NE * (4 / NW) * 8);
    m.seed_s = m.thr_s + 4 * NW * TILE;
    uint64_t* bars = reinterpret_cast<uint64_t*>(m.seed_s + NW * TILE);
    m.q_full = bars;
    m.k_full = bars + 1;
    m.k_empty = bars + 1 + MASK_S;
    m.s_full = bars + 1 + 2 * MASK_S;
    m.s_free = m.s_full + MASK_NB;
    m.fixed = m.s_free + MASK_NB;
    m.drain = m.fixed + 1;
    uint32_t* holder = reinterpret_cast<uint32_t*>(bars + 24);
    int* qidx_blk = reinterpret_cast<int*>(holder + 4);      // [128]
    int* misc = qidx_blk + TILE;                             // [8] warp counts, tile count
    uint32_t* sched = reinterpret_cast<uint32_t*>(misc + 16);   // [nKB]
    m.flags = reinterpret_cast<uint8_t*>(sched + s.nKB);
    m.qidx_blk = qidx_blk;
    m.sched = sched;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int2 bq = grid_order(s.BH, s.nQB, s.causal != 0);
    const int bh = bq.x, qb = bq.y;
    const int32_t* Kidx_bh = Kidx + (size_t)bh * s.NK;

    if (threadIdx.x == 0) {
        mask_init_barriers<MASK_NB>(m, NE);
        fence_barrier_init();
        // Q does not depend on the schedule built below: issue it now
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        mbar_expect_tx(m.q_full, TB);
        for (int bx = 0; bx < D / BOX; ++bx)
            tma_load_3d(m.sQ + bx * BOX_BYTES, &tmQ, m.q_full, bx * BOX, qb * TILE, bh);
    }
    if (warp == 1) { tmem_alloc(holder, 512); tmem_relinquish(); }
    if (threadIdx.x >= EPI0) {
        const int r = threadIdx.x - EPI0;
        if (r < TILE) {
            const int q = qb * TILE + r;
            qidx_blk[r] = (q < s.NQ && s.causal) ? Qidx[(size_t)bh * s.NQ + q] : INT_MAX;
        }
        for (int i = r; i < 4 * NW * TILE; i += NE) m.thr_s[i] = ASA_SENTINEL;
        for (int i = r; i < s.nKB; i += NE) m.flags[i] = 0;
        if (r < NEPI) {                       // the schedule builders' barrier counts NEPI threads
            const int n = sched_visible(sched, misc, s, bd, bh, qb, r);
            if (r == 0) misc[8] = n;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *holder;
    const int qmin_blk = s.causal ? bd.qmin[bh * s.nQB + qb] : INT_MIN;
    m.T = misc[8];

    if (warp == 0) {
        if (lane == 0) mask_produce<D>(m, &tmK, s, bh, err);
    } else if (warp == 1) {
        mask_mma<D>(m, s, tbase, lane, err);
    } else {
        const int row = (warp & 3) * 32 + lane;
        const int et = threadIdx.x - EPI0;
        const int q = qb * TILE + row;
        const bool qv = q < s.NQ;
        const int qpos = !qv ? INT_MIN : (s.causal ? Qidx[(size_t)bh * s.NQ + q] : INT_MAX);
        TopK<KM> tk;
        mask_epilogue<D, KM, NW>(m, s, Kidx_bh, qmin_blk, tbase, warp, lane, et, qpos, tk, err);
        float mv[KM];
        mask_merge<KM, NW>(m, s, tk, reinterpret_cast<unsigned long long*>(m.sK), row, et / TILE, qv,
                           (size_t)bh * s.NQ + (qv ? q : 0), topv, topi, mv);
        uint8_t* Mrow = M + ((size_t)bh * s.nQB + qb) * s.nKB;
        for (int i = et; i < s.nKB; i += NE) Mrow[i] = m.flags[i];
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
}

// ===========================================================================
// K1 exact: the exact α-entmax threshold (asa_tau_mode ASA_TAU_EXACT) and the
// "tile max vs τ" mask, no counterpart in the reference.  τ solves
// Σ_j [(α-1)s_j - τ]_+^{1/(α-1)} = 1 over every visible key of the row (s the
// clamped score).  kExactPasses passes over the row's visible tiles, S =
// Q·K^T on the tensor cores each time: the first finds the row maximum,
// which brackets τ in [(α-1)s_max - 1, (α-1)s_max]; each later pass sums
// F(τ) = Σ u_+^{1/(α-1)} and Σ u_+^{(2-α)/(α-1)} and takes a Newton step (F
// is convex and decreasing, so from the left end the steps climb
// monotonically), falling back to bisection when a step leaves the bracket.
// The row's NW threads (one per column slice) add their partial sums in a
// fixed order between passes, so every thread of a row holds the same τ.
// The last pass marks each tile holding a positive weight at the bracket's
// left end, which bounds the final τ from below: a superset of the tiles the
// final τ leaves weight in.
// ===========================================================================
template <int D, int NW, int PINV, int PE2>
__global__ void __launch_bounds__(64 + 128 * NW, 1)
k1_exact(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK, Shape s,
         const int32_t* __restrict__ Qidx, const int32_t* __restrict__ Kidx, Bounds bd,
         float* __restrict__ tau, uint8_t* __restrict__ M, int* err) {
    constexpr int NE = 128 * NW;              // epilogue threads
    constexpr int CP = 4 / NW;                // 32-column chunks per thread per tile
    constexpr int S = 4;                      // K stages
    constexpr int NB = 4;                     // S buffers in TMEM (128 columns each)
    constexpr int TB = D * TILE * 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = align1024(smem_raw, err);
    uint8_t* sQ = base;
    uint8_t* sK = base + TB;
    float* red = reinterpret_cast<float*>(sK + S * TB);    // [2 parities][2][NW][128] partial sums
    uint64_t* bars = reinterpret_cast<uint64_t*>(red + 4 * NW * TILE);
    uint64_t* q_full = bars;
    uint64_t* k_full = bars + 1;
    uint64_t* k_empty = k_full + S;
    uint64_t* s_full = k_empty + S;           // [NB]
    uint64_t* s_free = s_full + NB;           // [NB]
    uint64_t* drain = s_free + NB;            // exit-time MMA drain (after a timed-out wait)
    uint32_t* holder = reinterpret_cast<uint32_t*>(bars + 24);
    int* misc = reinterpret_cast<int*>(holder + 4);        // [8] warp counts, tile count
    uint32_t* sched = reinterpret_cast<uint32_t*>(misc + 16);   // [nKB]
    uint8_t* flags = reinterpret_cast<uint8_t*>(sched + s.nKB);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int2 bq = grid_order(s.BH, s.nQB, s.causal != 0);
    const int bh = bq.x, qb = bq.y;
    const int32_t* Kidx_bh = Kidx + (size_t)bh * s.NK;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < S; ++i) { mbar_init(&k_full[i], 1); mbar_init(&k_empty[i], 1); }
        for (int i = 0; i < NB; ++i) { mbar_init(&s_full[i], 1); mbar_init(&s_free[i], NE / 32); }
        mbar_init(drain, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        mbar_expect_tx(q_full, TB);
        for (int bx = 0; bx < D / BOX; ++bx)
            tma_load_3d(sQ + bx * BOX_BYTES, &tmQ, q_full, bx * BOX, qb * TILE, bh);
    }
    if (warp == 1) { tmem_alloc(holder, 512); tmem_relinquish(); }
    if (threadIdx.x >= EPI0) {
        const int r = threadIdx.x - EPI0;
        for (int i = r; i < s.nKB; i += NE) flags[i] = 0;
        if (r < NEPI) {                       // the schedule builders' barrier counts NEPI threads
            const int n = sched_visible(sched, misc, s, bd, bh, qb, r);
            if (r == 0) misc[8] = n;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *holder;
    const int T = misc[8];
    const int TP = kExactPasses * T;          // every pass: tile jj % T

    if (warp == 0) {
        if (lane == 0) {
            for (int j = 0; j < TP; ++j) {
                const int kb = (int)(sched[j % T] & SCHED_IDX);
                const int st = j % S;
                mbar_wait(&k_empty[st], ((j / S) & 1) ^ 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                mbar_expect_tx(&k_full[st], TB);
                for (int bx = 0; bx < D / BOX; ++bx)
                    tma_load_3d(sK + st * TB + bx * BOX_BYTES, &tmK, &k_full[st], bx * BOX, kb * TILE, bh);
            }
        }
        if (lane == 0 && error_set(err)) {   // a wait gave up: let this CTA's loads land
            mbar_drain(q_full, 0);
            drain_ring(k_full, S, TP);
        }
    } else if (warp == 1) {
        constexpr uint32_t idesc = idesc_bf16(128, 128, 0, 0);
        mbar_wait(q_full, 0, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);   // issued at set-up even when T = 0
        const uint64_t dQd = kdesc(sQ, 0);
        for (int j = 0; j < TP; ++j) {
            const int st = j % S, b = j % NB;
            mbar_wait(&k_full[st], (j / S) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            mbar_wait(&s_free[b], ((j / NB) & 1) ^ 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            tc_fence_after();
            if (lane == 0) {
                const uint64_t dK = kdesc(sK + st * TB, 0);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk)
                    mma_bf16_ss(tbase + b * 128, kdesc_step(dQd, kk), kdesc_step(dK, kk), idesc, kk > 0);
                mma_commit(&s_full[b]);
                mma_commit(&k_empty[st]);
            }
            __syncwarp();
        }
        if (lane == 0 && error_set(err)) {   // a wait gave up: let this CTA's MMAs finish
            mma_commit(drain);
            mbar_drain(drain, 0);
        }
        __syncwarp();
    } else {
        const int row = (warp & 3) * 32 + lane;
        const int et = threadIdx.x - EPI0;
        const int h = et / TILE;                  // column slice of each tile
        const int q = qb * TILE + row;
        const bool qv = q < s.NQ;
        const int qpos = !qv ? INT_MIN : (s.causal ? Qidx[(size_t)bh * s.NQ + q] : INT_MAX);
        const uint32_t tl = tmem_lane_base(tbase, warp);
        const float inv = __fdiv_rn(1.0f, s.am1);
        float tq = 0.0f, lo = 0.0f, hi = 0.0f;    // τ and its bracket (identical in the row's threads)
        float a0 = neg_inf(), a1 = 0.0f;          // this pass's partials: max, or F and Σ w
        // add the row's partial sums (fixed order: deterministic), then step τ
        auto combine = [&](int pass) {
            float* rp = red + (pass & 1) * 2 * NW * TILE;
            rp[h * TILE + row] = a0;
            rp[(NW + h) * TILE + row] = a1;
            asm volatile("bar.sync 2, %0;" ::"n"(NE) : "memory");
            if (pass == 0) {
                float m = neg_inf();
#pragma unroll
                for (int g = 0; g < NW; ++g) m = fmaxf(m, rp[g * TILE + row]);
                if (!(m > neg_inf())) m = 0.0f;       // no visible key: no weight anywhere
                hi = __fmul_rn(s.am1, m);             // m is a clamped score
                lo = __fadd_rn(hi, -1.0f);
                tq = lo;
            } else {
                float F = 0.0f, W = 0.0f;
#pragma unroll
                for (int g = 0; g < NW; ++g) {
                    F += rp[g * TILE + row];
                    W += rp[(NW + g) * TILE + row];
                }
                const float gF = F - 1.0f;
                if (gF >= 0.0f) lo = tq; else hi = tq;
                float tn = W > 0.0f ? tq + gF / (inv * W) : tq;
                if (!(tn >= lo && tn <= hi)) tn = 0.5f * (lo + hi);
                tq = tn;
            }
            a0 = 0.0f;
            a1 = 0.0f;
        };
        for (int jj = 0; jj < TP; ++jj) {
            const int pass = jj / T;
            if (jj > 0 && jj % T == 0) combine(pass - 1);
            const bool last = pass == kExactPasses - 1;
            const uint32_t e = sched[jj % T];
            const int kb = (int)(e & SCHED_IDX);
            const int b = jj % NB;
            const bool all = (e & SCHED_ALL) != 0;
            mbar_wait(&s_full[b], (jj / NB) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            tc_fence_after();
            uint32_t r2[CP][32];
#pragma unroll
            for (int cc = 0; cc < CP; ++cc) tmem_ld32(tl + b * 128 + (h * CP + cc) * 32, r2[cc]);
            tmem_ld_wait();
            tc_fence_before();
            epi_arrive(&s_free[b]);          // S is in registers: release the buffer
            bool hit = false;
#pragma unroll
            for (int cc = 0; cc < CP; ++cc) {
                const uint32_t vis = all ? 0xffffffffu
                                         : vis_mask32(Kidx_bh, kb * TILE + (h * CP + cc) * 32, s.NK, s.causal, qpos);
                if (pass == 0) {
                    // the clamp is monotone for scale > 0: clamp the chunk's
                    // largest raw score; otherwise clamp each
                    if (s.scale > 0.0f) {
                        uint32_t r[32];
#pragma unroll
                        for (int i = 0; i < 32; ++i) r[i] = ((vis >> i) & 1u) ? r2[cc][i] : 0xff800000u;
                        float gm[11];
                        const float cm = chunk_max(r, gm);
                        if (cm > neg_inf()) a0 = fmaxf(a0, clamp_score(cm, s.scale));
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if ((vis >> i) & 1u) a0 = fmaxf(a0, clamp_score(__uint_as_float(r2[cc][i]), s.scale));
                    }
                    continue;
                }
                exact_sums<PINV, PE2>(r2[cc], vis, s, tq, lo, last, a0, a1, hit);
            }
            if (hit) flags[kb] = 1;
        }
        if (T > 0) combine(kExactPasses - 1);
        if (h == 0 && qv) tau[(size_t)bh * s.NQ + q] = T > 0 ? tq : 0.0f;
        asm volatile("bar.sync 2, %0;" ::"n"(NE) : "memory");
        uint8_t* Mrow = M + ((size_t)bh * s.nQB + qb) * s.nKB;
        for (int i = et; i < s.nKB; i += NE) Mrow[i] = flags[i];
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
}

// Coalesced store of a warp's 32 rows x 32 columns (lane i holds row i's
// values o[0..31]) through 4 KB of shared staging: row-per-lane stores write
// 32 different lines per instruction, partial sectors that cost more than
// the whole tile's MMAs.  Rows at or beyond nrows are skipped.
template <typename TO>
__device__ __forceinline__ void warp_store_rows(TO* base, int ld, int nrows, int col0, const float (&o)[32],
                                                float* stage, int lane) {
#pragma unroll
    for (int i = 0; i < 32; ++i) stage[lane * 33 + i] = o[i];
    __syncwarp();
    if constexpr (sizeof(TO) == 4) {
#pragma unroll 4
        for (int r = 0; r < 32; ++r)
            if (r < nrows) base[(size_t)r * ld + col0 + lane] = stage[r * 33 + lane];
    } else {
        const int cc = (lane & 15) * 2;
#pragma unroll 4
        for (int r2 = 0; r2 < 16; ++r2) {
            const int r = 2 * r2 + (lane >> 4);
            if (r < nrows)
                *reinterpret_cast<uint32_t*>(base + (size_t)r * ld + col0 + cc) =
                    pack_bf16(stage[r * 33 + cc], stage[r * 33 + cc + 1]);
        }
    }
    __syncwarp();
}

// A warp's 32 rows x 32 columns (lane = row, values o[0..31]) staged in
// shared memory in the store maps' swizzled layouts -- fp32 rows of 128 B
// (16-byte chunk j of row r at j ^ (r & 7)), bf16 rows of 64 B (chunk j at
// j ^ ((r >> 1) & 3)) -- and written by TMA: to mA (fp32) when wA, to mB
// when wB (fp32 from the same staging if B16 is false, else bf16).  stage:
// 6 KB, 1024-byte aligned; the caller waits (bulk_wait_read) before reusing
// it.  Rows past the tensor's end are clipped by the TMA unit.
template <bool B16>
__device__ __forceinline__ void warp_tma_store(const CUtensorMap* mA, bool wA, const CUtensorMap* mB, bool wB,
                                               uint8_t* stage, const float (&o)[32], int lane, int x, int y,
                                               int z) {
    if (wA || (wB && !B16)) {
        float4* st = reinterpret_cast<float4*>(stage);
#pragma unroll
        for (int j = 0; j < 8; ++j)
            st[lane * 8 + (j ^ (lane & 7))] = make_float4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
    }
    if (wB && B16) {
        uint4* st = reinterpret_cast<uint4*>(stage + 4096);
#pragma unroll
        for (int j = 0; j < 4; ++j)
            st[lane * 4 + (j ^ ((lane >> 1) & 3))] =
                make_uint4(pack_bf16(o[8 * j], o[8 * j + 1]), pack_bf16(o[8 * j + 2], o[8 * j + 3]),
                           pack_bf16(o[8 * j + 4], o[8 * j + 5]), pack_bf16(o[8 * j + 6], o[8 * j + 7]));
    }
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
        if (wA) tma_store_3d(mA, stage, x, y, z);
        if (wB) tma_store_3d(mB, B16 ? stage + 4096 : stage, x, y, z);
        bulk_commit();
    }
    __syncwarp();
}

// Store this thread's fp32 values o[0..31] (columns [32c, 32c+32) of `row`)
// to a row-major [rows][D] output of type TO.
template <int D, typename TO>
__device__ __forceinline__ void store_out32(TO* dst_row, int c, const float (&o)[32]) {
    if constexpr (sizeof(TO) == 2) {
        uint4* dst = reinterpret_cast<uint4*>(dst_row + c * 32);
#pragma unroll
        for (int i = 0; i < 4; ++i)
            dst[i] = make_uint4(pack_bf16(o[8 * i], o[8 * i + 1]), pack_bf16(o[8 * i + 2], o[8 * i + 3]),
                                pack_bf16(o[8 * i + 4], o[8 * i + 5]), pack_bf16(o[8 * i + 6], o[8 * i + 7]));
    } else {
        float4* dst = reinterpret_cast<float4*>(dst_row + c * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
    }
}

// ===========================================================================
// K3: forward over the CSR tile list
// ===========================================================================
// Shared memory: Q, three K stages (released once S = Q·K^T completes) and
// two V stages (released after P·V), loaded by separate producer threads.
// TMEM: three S buffers (columns 0-383) and O (384-511).  The epilogue
// writes P back over its own S columns as bf16 hi/lo pairs (each 16-key
// group: 8 hi columns then 8 lo columns), which the tensor cores read as the
// A operand of O += P·V; a buffer is reused once that P·V completes.  The MMA
// warp issues S two tiles ahead of the P·V it waits for.  NW epilogue
// warpgroups split each tile by columns (128/NW per thread).
//
// Written as role functions over a shared-memory view, shared by the
// stand-alone forward and the fused τ/mask + forward kernel.
constexpr int FWD_S = 3;     // K stages
constexpr int FWD_SV = 2;    // V stages
constexpr int FWD_NB = 3;    // S / P buffers in TMEM
constexpr uint32_t FWD_TO = 384;   // TMEM column of O

struct FwdPhase {
    uint8_t* sQ;
    uint8_t* sK;              // FWD_S stages
    uint8_t* sV;              // FWD_SV stages
    uint64_t* k_full;
    uint64_t* k_empty;
    uint64_t* v_full;
    uint64_t* v_empty;
    uint64_t* s_full;         // [FWD_NB]
    uint64_t* s_free;         // [FWD_NB]
    uint64_t* p_full;         // [FWD_NB]
    uint64_t* o_full;
    uint64_t* fixed;          // K/V of a tile-load-zeroing tile fixed
    uint64_t* drain;          // [2] exit-time MMA drains (after a timed-out wait)
    float* nsum;              // [NW][128] partial row sums
    const int* qidx_blk;
    const uint32_t* sched;    // [T] active key blocks
    int T;
};
constexpr int FWD_BARS = 2 * FWD_S + 2 * FWD_SV + 3 * FWD_NB + 4;

// Barriers start at `bars` (FWD_BARS of them); epilogue warps ew arrive.
__device__ __forceinline__ void fwd_init_barriers(FwdPhase& f, uint64_t* bars, int ew) {
    f.k_full = bars;
    f.k_empty = f.k_full + FWD_S;
    f.v_full = f.k_empty + FWD_S;
    f.v_empty = f.v_full + FWD_SV;
    f.s_full = f.v_empty + FWD_SV;
    f.s_free = f.s_full + FWD_NB;
    f.p_full = f.s_free + FWD_NB;
    f.o_full = f.p_full + FWD_NB;
    f.fixed = f.o_full + 1;
    f.drain = f.fixed + 1;
    if (threadIdx.x == 0) {
        for (int i = 0; i < FWD_S; ++i) { mbar_init(&f.k_full[i], 1); mbar_init(&f.k_empty[i], 1); }
        for (int i = 0; i < FWD_SV; ++i) { mbar_init(&f.v_full[i], 1); mbar_init(&f.v_empty[i], 1); }
        for (int i = 0; i < FWD_NB; ++i) {
            mbar_init(&f.s_full[i], 1); mbar_init(&f.s_free[i], 1); mbar_init(&f.p_full[i], ew);
        }
        mbar_init(f.o_full, 1);
        mbar_init(f.fixed, ew);
        mbar_init(&f.drain[0], 1);
        mbar_init(&f.drain[1], 1);
    }
}

// Producers: lane 0 the K ring, lane 1 the V ring (V's ring, freed after
// P·V, must not hold back K's, freed after S), from tile j0 on (tiles before
// it were issued at set-up).
template <int D>
__device__ void fwd_produce(const FwdPhase& f, const CUtensorMap* tmK, const CUtensorMap* tmV, const Shape& s,
                            int bh, int lane, int j0, const uint64_t* q_full, int* err) {
    constexpr int TB = D * TILE * 2;
    if (lane == 0) {
        for (int j = j0; j < f.T; ++j) {
            const int kb = (int)(f.sched[j] & SCHED_IDX);
            const int st = j % FWD_S;
            mbar_wait(&f.k_empty[st], ((j / FWD_S) & 1) ^ 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            mbar_expect_tx(&f.k_full[st], TB);
            for (int bx = 0; bx < D / BOX; ++bx)
                tma_load_3d(f.sK + st * TB + bx * BOX_BYTES, tmK, &f.k_full[st], bx * BOX, kb * TILE, bh);
        }
    } else if (lane == 1) {
        for (int j = j0; j < f.T; ++j) {
            const int kb = (int)(f.sched[j] & SCHED_IDX);
            const int sv = j % FWD_SV;
            mbar_wait(&f.v_empty[sv], ((j / FWD_SV) & 1) ^ 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            mbar_expect_tx(&f.v_full[sv], TB);
            for (int bx = 0; bx < D / BOX; ++bx)
                tma_load_3d(f.sV + sv * TB + bx * BOX_BYTES, tmV, &f.v_full[sv], bx * BOX, kb * TILE, bh);
        }
    }
    __syncwarp();
    if (lane == 0 && f.T > 0 && error_set(err)) {   // a wait gave up: let this CTA's loads land
        if (q_full) mbar_drain(const_cast<uint64_t*>(q_full), 0);
        drain_ring(f.k_full, FWD_S, f.T);
        drain_ring(f.v_full, FWD_SV, f.T);
    }
}

// S = Q·K^T issuer.  tcgen05.mma issue blocks at the tensor pipe's rate, so
// S and P·V come from two warps: while one waits for its inputs the other
// keeps the pipe fed.  S(n) needs its K tile and TMEM buffer n % NB, which
// P·V(n - NB) frees.  q_full: the Q barrier to wait on first, or null when
// Q is known to be resident.
template <int D>
__device__ void fwd_mma_s(const FwdPhase& f, const Shape& s, uint32_t tbase, int lane, uint64_t* q_full,
                          int* err) {
    constexpr int TB = D * TILE * 2;
    constexpr uint32_t idS = idesc_bf16(128, 128, 0, 0);
    if (f.T > 0 && q_full) mbar_wait(q_full, 0, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
    const uint64_t dQ = kdesc(f.sQ, 0);
    int nfix = 0;
    for (int n = 0; n < f.T; ++n) {
        const uint32_t e = f.sched[n];
        const int st = n % FWD_S, b = n % FWD_NB;
        uint8_t* kt = f.sK + st * TB;
        mbar_wait(&f.k_full[st], (n / FWD_S) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
        if (e & SCHED_FIX)     // the epilogue warps zero K and V of this tile
            mbar_wait(f.fixed, (nfix++) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
        __syncwarp();
        mbar_wait(&f.s_free[b], ((n / FWD_NB) & 1) ^ 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
        tc_fence_after();
        if (lane == 0) {
            const uint64_t dK = kdesc(kt, 0);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk)
                mma_bf16_ss(tbase + b * 128, kdesc_step(dQ, kk), kdesc_step(dK, kk), idS, kk > 0);
            mma_commit(&f.s_full[b]);
            mma_commit(&f.k_empty[st]);
        }
        __syncwarp();
    }
    if (lane == 0 && error_set(err)) {   // a wait gave up: let this warp's MMAs finish
        mma_commit(&f.drain[0]);
        mbar_drain(&f.drain[0], 0);
    }
    __syncwarp();
}

// O += P·V issuer: P·V(m) needs its V tile and the epilogue's P.  P·V(m)
// needs no wait on `fixed`: p_full(m) completes only after every epilogue
// warp's arrival, and the warps that zero V of a tile-load-zeroing tile
// arrive after that zeroing and its proxy fence.
template <int D>
__device__ void fwd_mma_pv(const FwdPhase& f, const Shape& s, uint32_t tbase, int lane, int split, int* err) {
    constexpr int TB = D * TILE * 2;
    constexpr uint32_t idPV = idesc_bf16(128, D, 0, 1);
    for (int m = 0; m < f.T; ++m) {
        const int b = m % FWD_NB, sv = m % FWD_SV;
        uint8_t* vt = f.sV + sv * TB;
        mbar_wait(&f.v_full[sv], (m / FWD_SV) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
        __syncwarp();
        mbar_wait(&f.p_full[b], (m / FWD_NB) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
        tc_fence_after();
        if (lane == 0) {
            const uint32_t pb = tbase + b * 128;
            const uint64_t dV = mndesc(vt, 0);
#pragma unroll
            for (int kk = 0; kk < TILE / 16; ++kk)
                mma_bf16_ts(tbase + FWD_TO, pb + kk * 16, mndesc_step(dV, kk), idPV, (m > 0 || kk > 0));
            if (split) {
#pragma unroll
                for (int kk = 0; kk < TILE / 16; ++kk)
                    mma_bf16_ts(tbase + FWD_TO, pb + kk * 16 + 8, mndesc_step(dV, kk), idPV, 1);
            }
            mma_commit(&f.s_free[b]);
            mma_commit(&f.v_empty[sv]);
        }
        __syncwarp();
    }
    if (lane == 0) mma_commit(f.o_full);
    if (lane == 0 && error_set(err)) {   // a wait gave up: let this warp's MMAs finish
        mma_commit(&f.drain[1]);
        mbar_drain(&f.drain[1], 0);
    }
    __syncwarp();
}

// Epilogue thread et (row = TMEM lane, column slice h = et / 128): entmax
// weights of every scheduled tile written back to TMEM as P, the row sum,
// then O / (n + EPS) stored (fp32 copy O32 and/or O in TO).  tq: the row's τ.
template <int D, typename TO, int PINV, int NW>
__device__ void fwd_epilogue(const FwdPhase& f, const Shape& s, const int32_t* __restrict__ Kidx_bh,
                             int qmin_blk, uint32_t tbase, int warp, int lane, int et, int bh, int qb,
                             int qpos, float tq, TO* __restrict__ O, float* __restrict__ O32,
                             const CUtensorMap* mO32, const CUtensorMap* mO, float* __restrict__ rownorm,
                             int split, int* err) {
    constexpr int NE = 128 * NW;
    constexpr int CP = 4 / NW;                // 32-column chunks per thread per tile
    constexpr int TB = D * TILE * 2;
    const int row = (warp & 3) * 32 + lane;
    const int h = et / TILE;
    const int q = qb * TILE + row;
    const bool qv = q < s.NQ;
    const size_t qrow = (size_t)bh * s.NQ + (qv ? q : 0);
    const uint32_t tl = tmem_lane_base(tbase, warp);
    float n = 0.0f;
    constexpr bool kPacked = PINV == 1 || PINV == 2 || PINV == 4;
    const float2 c1 = make_float2(__fmul_rn(s.am1, s.scale), __fmul_rn(s.am1, s.scale));
    const float2 mtau = make_float2(-tq, -tq);
    const float uhi = __fmaf_rn(s.am1, 10.0f, -tq);
    // warp-uniform: the packed path issues warp-collective TMEM loads/stores
    const bool packed_row = __all_sync(0xffffffffu, kPacked && split && __fmaf_rn(s.am1, -10.0f, -tq) <= 0.0f);
    float2 n2 = make_float2(0.0f, 0.0f);
    for (int j = 0; j < f.T; ++j) {
        const uint32_t e = f.sched[j];
        const int kb = (int)(e & SCHED_IDX);
        const bool all = (e & SCHED_ALL) != 0;
        const int b = j % FWD_NB;
        if (e & SCHED_FIX) {
            // The reference's tile-load zeroing of this tile's K and V, by
            // eight epilogue warps (32 rows each of K or V) instead of one
            // control warp: S and P·V wait for it.
            const int ew = et >> 5;
            if (ew < 8) {
                uint8_t* tile;
                if (ew < 4) {
                    mbar_wait(&f.k_full[j % FWD_S], (j / FWD_S) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                    tile = f.sK + (j % FWD_S) * TB;
                } else {
                    mbar_wait(&f.v_full[j % FWD_SV], (j / FWD_SV) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                    tile = f.sV + (j % FWD_SV) * TB;
                }
                fix_tile<D, 1>(tile, f.qidx_blk, qmin_blk, Kidx_bh, kb, s.NK, lane, 32 * (ew & 3));
                fence_async_smem();
            }
            epi_arrive(f.fixed);
        }
        mbar_wait(&f.s_full[b], (j / FWD_NB) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
        tc_fence_after();
        if (kPacked && packed_row) {
            // the thread's chunks loaded at once, packed math; on partially
            // visible tiles invisible keys are masked to p = 0
            uint32_t r[CP][32];
#pragma unroll
            for (int cc = 0; cc < CP; ++cc) tmem_ld32(tl + b * 128 + (h * CP + cc) * 32, r[cc]);
            uint32_t vis[CP];
#pragma unroll
            for (int cc = 0; cc < CP; ++cc)
                vis[cc] = all ? 0xffffffffu : vis_mask32(Kidx_bh, kb * TILE + (h * CP + cc) * 32, s.NK, s.causal, qpos);
            tmem_ld_wait();
            // fully visible tiles (almost all) skip the per-key visibility select
            auto weights = [&](auto all_vis) {
#pragma unroll
                for (int cc = 0; cc < CP; ++cc) {
                    const uint32_t col = tl + b * 128 + (h * CP + cc) * 32;
#pragma unroll
                    for (int g = 0; g < 2; ++g) {
                        uint32_t hi[8], lo[8];
#pragma unroll
                        for (int m = 0; m < 8; ++m) {
                            float2 pp = entmax_pair<PINV>(r[cc][16 * g + 2 * m], r[cc][16 * g + 2 * m + 1],
                                                          c1, mtau, uhi);
                            if constexpr (!decltype(all_vis)::value) {
                                const int bit = 16 * g + 2 * m;
                                pp.x = (vis[cc] >> bit) & 1u ? pp.x : 0.0f;
                                pp.y = (vis[cc] >> (bit + 1)) & 1u ? pp.y : 0.0f;
                            }
                            n2 = __fadd2_rn(n2, pp);
                            split_pair(pp, hi[m], lo[m]);
                        }
                        tmem_st8(col + g * 16, hi);
                        tmem_st8(col + g * 16 + 8, lo);
                    }
                }
            };
            if (all) weights(std::true_type{});
            else weights(std::false_type{});
            tmem_st_wait();
            tc_fence_before();
            epi_arrive(&f.p_full[b]);
            continue;
        }
#pragma unroll
        for (int cc = 0; cc < CP; ++cc) {
            const int c = h * CP + cc;
            uint32_t r[32];
            tmem_ld32(tl + b * 128 + c * 32, r);
            tmem_ld_wait();
            float p[32];
            if (all) {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float u = __fmaf_rn(s.am1, clamp_score(__uint_as_float(r[i]), s.scale), -tq);
                    p[i] = entmax_pk<PINV>(u, s.pinv.e);
                    n += p[i];
                }
            } else {
                const uint32_t vis = vis_mask32(Kidx_bh, kb * TILE + c * 32, s.NK, s.causal, qpos);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const bool v = (vis >> i) & 1u;
                    const float u = __fmaf_rn(s.am1, clamp_score(__uint_as_float(r[i]), s.scale), -tq);
                    p[i] = v ? entmax_pk<PINV>(u, s.pinv.e) : 0.0f;
                    n += p[i];
                }
            }
            // two 16-key groups: hi then lo columns over the group's own S columns
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                uint32_t hi[8], lo[8];
#pragma unroll
                for (int m = 0; m < 8; ++m) {
                    const float x0 = p[16 * g + 2 * m], x1 = p[16 * g + 2 * m + 1];
                    const __nv_bfloat162 hh = __floats2bfloat162_rn(x0, x1);
                    const float2 hf = __bfloat1622float2(hh);
                    hi[m] = *reinterpret_cast<const uint32_t*>(&hh);
                    lo[m] = pack_bf16(x0 - hf.x, x1 - hf.y);
                }
                tmem_st8(tl + b * 128 + c * 32 + g * 16, hi);
                if (split) tmem_st8(tl + b * 128 + c * 32 + g * 16 + 8, lo);
            }
        }
        tmem_st_wait();
        tc_fence_before();
        epi_arrive(&f.p_full[b]);
    }
    n += n2.x + n2.y;
    // row sum: the warpgroups' partial sums added in group order
    f.nsum[h * TILE + row] = n;
    asm volatile("bar.sync 2, %0;" ::"n"(NE) : "memory");
    if (h == 0) {
        for (int g = 1; g < NW; ++g) n += f.nsum[g * TILE + row];
        if (qv) rownorm[qrow] = n;
        f.nsum[row] = n;
    }
    asm volatile("bar.sync 2, %0;" ::"n"(NE) : "memory");
    n = f.nsum[row];
    mbar_wait(f.o_full, 0, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
    tc_fence_after();
    const float inv = __fdiv_rn(1.0f, __fadd_rn(n, ASA_EPS));
    // every MMA is done: the K stages are free for the store staging (6 KB
    // per storing warp: at most 16 warps x 6 KB = the three K stages at
    // D = 128; at D = 64 only the first eight warps store)
    uint8_t* stage = f.sK + (et >> 5) * 6144;
    const int q0 = qb * TILE + (warp & 3) * 32;
    const int nrows = min(32, s.NQ - q0);
    const bool wA = O32 != nullptr, wB = sizeof(TO) == 2 || (void*)O != (void*)O32;
    bool pending = false;
#pragma unroll 1
    for (int c = h; c < D / 32; c += NW) {
        uint32_t r[32];
        tmem_ld32(tl + FWD_TO + c * 32, r);
        tmem_ld_wait();
        if (nrows <= 0) continue;
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            float v = f.T > 0 ? __uint_as_float(r[i]) * inv : 0.0f;
            o[i] = isfinite(v) ? v : 0.0f;
        }
        if (pending) {   // the previous chunk's stores have read the staging
            if (lane == 0) bulk_wait_read();
            __syncwarp();
        }
        warp_tma_store<sizeof(TO) == 2>(mO32, wA, mO, wB, stage, o, lane, c * 32, q0, bh);
        pending = true;
    }
    if (pending && lane == 0) bulk_wait_read();   // before the CTA's shared memory is released
    __syncwarp();
}

template <int NW>
constexpr int fwd_threads() { return K3_EPI0 + 128 * NW; }

template <int D, typename TO, int PINV, int NW>
__global__ void __launch_bounds__(fwd_threads<NW>(), 1)
k3_forward(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
           const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO32,
           const __grid_constant__ CUtensorMap tmO, Shape s, const int32_t* __restrict__ Qidx,
           const int32_t* __restrict__ Kidx, Bounds bd, const float* __restrict__ tau,
           const int32_t* __restrict__ ptr, const int32_t* __restrict__ idx, TO* __restrict__ O,
           float* __restrict__ O32, float* __restrict__ rownorm, int split, int* err) {
    constexpr int TB = D * TILE * 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = align1024(smem_raw, err);
    FwdPhase f;
    f.sQ = base;
    f.sK = base + TB;
    f.sV = f.sK + FWD_S * TB;
    uint64_t* bars = reinterpret_cast<uint64_t*>(f.sV + FWD_SV * TB);
    uint64_t* q_full = bars;
    uint32_t* holder = reinterpret_cast<uint32_t*>(bars + 24);
    f.nsum = reinterpret_cast<float*>(holder + 4);                    // [NW][128]
    int* qidx_blk = reinterpret_cast<int*>(f.nsum + NW * TILE);       // [128]
    uint32_t* sched = reinterpret_cast<uint32_t*>(qidx_blk + TILE);   // [T]
    f.qidx_blk = qidx_blk;
    f.sched = sched;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int2 bq = grid_order(s.BH, s.nQB, s.causal != 0);
    const int bh = bq.x, qb = bq.y;
    const int32_t* Kidx_bh = Kidx + (size_t)bh * s.NK;
    const int32_t* list = idx + (size_t)bh * s.nQB * s.nKB;
    const int e0 = ptr[(size_t)bh * (s.nQB + 1) + qb];
    f.T = ptr[(size_t)bh * (s.nQB + 1) + qb + 1] - e0;

    fwd_init_barriers(f, bars + 1, 4 * NW);
    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        fence_barrier_init();
        if (f.T > 0) {
            // Q and the first K/V tiles do not depend on the schedule being
            // built below: issue them now so their latency hides the set-up
            const int kb0 = list[e0];
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            mbar_expect_tx(q_full, TB);
            mbar_expect_tx(&f.k_full[0], TB);
            mbar_expect_tx(&f.v_full[0], TB);
            for (int bx = 0; bx < D / BOX; ++bx) {
                tma_load_3d(f.sQ + bx * BOX_BYTES, &tmQ, q_full, bx * BOX, qb * TILE, bh);
                tma_load_3d(f.sK + bx * BOX_BYTES, &tmK, &f.k_full[0], bx * BOX, kb0 * TILE, bh);
                tma_load_3d(f.sV + bx * BOX_BYTES, &tmV, &f.v_full[0], bx * BOX, kb0 * TILE, bh);
            }
        }
    }
    if (warp == 1) { tmem_alloc(holder, 512); tmem_relinquish(); }
    if (threadIdx.x >= K3_EPI0) {
        const int r = threadIdx.x - K3_EPI0;
        const int q = qb * TILE + r;
        if (r < TILE) qidx_blk[r] = (q < s.NQ && s.causal) ? Qidx[(size_t)bh * s.NQ + q] : INT_MAX;
        if (r < NEPI) sched_from_list(sched, list + e0, f.T, s, bd, bh, qb, false, r);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *holder;
    const int qmin_blk = s.causal ? bd.qmin[bh * s.nQB + qb] : INT_MIN;

    if (warp == 0) {
        fwd_produce<D>(f, &tmK, &tmV, s, bh, lane, 1, q_full, err);
    } else if (warp == 1) {
        fwd_mma_s<D>(f, s, tbase, lane, q_full, err);
    } else if (warp == 2) {
        fwd_mma_pv<D>(f, s, tbase, lane, split, err);
    } else {
        const int row = (warp & 3) * 32 + lane;
        const int et = threadIdx.x - K3_EPI0;
        const int q = qb * TILE + row;
        const bool qv = q < s.NQ;
        const size_t qrow = (size_t)bh * s.NQ + (qv ? q : 0);
        const int qpos = !qv ? INT_MIN : (s.causal ? Qidx[qrow] : INT_MAX);
        const float tq = qv ? tau[qrow] : 0.0f;
        fwd_epilogue<D, TO, PINV, NW>(f, s, Kidx_bh, qmin_blk, tbase, warp, lane, et, bh, qb, qpos, tq, O, O32,
                                      &tmO32, &tmO, rownorm, split, err);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
}

// ===========================================================================
// K13: the fused forward -- τ / mask and the forward in one CTA per query
// block (no counterpart in the reference, whose forward is three launches).
// Phase A is the τ / mask pass over the visible tiles; its merge yields the
// row's top-k, τ (solved by the row's merging thread with the same solve as
// k1_tau_solve), and the block's active key blocks, which become phase B's
// schedule directly: no tile lists are read, and Q stays in shared memory.
// Phase B's loads and S MMAs start while the τ solves run; its epilogue
// waits for τ.  TMEM: four S buffers in phase A, three S buffers and O in
// phase B.  Shared memory: Q, three K stages, then phase A's chunk copies
// and bounds, over which phase B's two V stages are laid.
// ===========================================================================
template <int D, int NW>
constexpr size_t fused_region_bytes() {
    return mask_extra_bytes<D, NW>() > (size_t)FWD_SV * D * TILE * 2 ? mask_extra_bytes<D, NW>()
                                                                      : (size_t)FWD_SV * D * TILE * 2;
}

template <int D, typename TO, int KM, int PINV, int NW>
__global__ void __launch_bounds__(fwd_threads<NW>(), 1)
k13_fused(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
          const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO32,
          const __grid_constant__ CUtensorMap tmO, Shape s, const int32_t* __restrict__ Qidx,
          const int32_t* __restrict__ Kidx, Bounds bd, float* __restrict__ tau, uint8_t* __restrict__ M,
          TO* __restrict__ O, float* __restrict__ O32, float* __restrict__ rownorm, int split, int* err) {
    constexpr int NE = 128 * NW;
    constexpr int TB = D * TILE * 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = align1024(smem_raw, err);
    MaskPhase m;
    FwdPhase f;
    m.sQ = f.sQ = base;
    m.sK = f.sK = base + TB;
    uint8_t* region = base + TB + MASK_S * TB;
    m.cbuf = reinterpret_cast<float4*>(region);
    m.thr_s = reinterpret_cast<float*>(m.cbuf + NE * (4 / NW) * 8);
    m.seed_s = m.thr_s + 4 * NW * TILE;
    f.sV = region;
    uint64_t* bars = reinterpret_cast<uint64_t*>(region + fused_region_bytes<D, NW>());
    m.q_full = bars;
    m.k_full = bars + 1;
    m.k_empty = bars + 1 + MASK_S;
    m.s_full = bars + 1 + 2 * MASK_S;
    m.s_free = m.s_full + MASK_NB;
    m.fixed = m.s_free + MASK_NB;
    m.drain = m.fixed + 1;
    uint64_t* fbars = bars + 24;                                        // FWD_BARS
    uint32_t* holder = reinterpret_cast<uint32_t*>(bars + 48);
    f.nsum = reinterpret_cast<float*>(holder + 4);                      // [NW][128]
    float* tau_s = f.nsum + NW * TILE;                                  // [128]
    int* qidx_blk = reinterpret_cast<int*>(tau_s + TILE);               // [128]
    int* misc = qidx_blk + TILE;                                        // [16]
    uint32_t* sched_a = reinterpret_cast<uint32_t*>(misc + 16);         // [nKB]
    uint32_t* sched_b = sched_a + s.nKB;                                // [nKB]
    m.flags = reinterpret_cast<uint8_t*>(sched_b + s.nKB);              // [nKB]
    m.qidx_blk = f.qidx_blk = qidx_blk;
    m.sched = sched_a;
    f.sched = sched_b;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int2 bq = grid_order(s.BH, s.nQB, s.causal != 0);
    const int bh = bq.x, qb = bq.y;
    const int32_t* Kidx_bh = Kidx + (size_t)bh * s.NK;

    fwd_init_barriers(f, fbars, 4 * NW);
    if (threadIdx.x == 0) {
        mask_init_barriers<MASK_NB>(m, NE);
        fence_barrier_init();
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        mbar_expect_tx(m.q_full, TB);
        for (int bx = 0; bx < D / BOX; ++bx)
            tma_load_3d(m.sQ + bx * BOX_BYTES, &tmQ, m.q_full, bx * BOX, qb * TILE, bh);
    }
    if (warp == 1) { tmem_alloc(holder, 512); tmem_relinquish(); }
    if (threadIdx.x >= K3_EPI0) {
        const int r = threadIdx.x - K3_EPI0;
        if (r < TILE) {
            const int q = qb * TILE + r;
            qidx_blk[r] = (q < s.NQ && s.causal) ? Qidx[(size_t)bh * s.NQ + q] : INT_MAX;
        }
        for (int i = r; i < 4 * NW * TILE; i += NE) m.thr_s[i] = ASA_SENTINEL;
        for (int i = r; i < s.nKB; i += NE) m.flags[i] = 0;
        if (r < NEPI) {                       // the schedule builders' barrier counts NEPI threads
            const int n = sched_visible(sched_a, misc, s, bd, bh, qb, r);
            if (r == 0) misc[8] = n;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *holder;
    const int qmin_blk = s.causal ? bd.qmin[bh * s.nQB + qb] : INT_MIN;
    m.T = misc[8];

    // ---- phase A: top-k and the block's active key blocks
    const int row = (warp & 3) * 32 + lane;
    const int et = threadIdx.x - K3_EPI0;
    const int q = qb * TILE + row;
    const bool qv = q < s.NQ;
    const size_t qrow = (size_t)bh * s.NQ + (qv ? q : 0);
    const int qpos = !qv ? INT_MIN : (s.causal ? Qidx[qrow] : INT_MAX);
    float mv[KM];
    if (warp == 0) {
        if (lane == 0) mask_produce<D>(m, &tmK, s, bh, err);
    } else if (warp == 1) {
        mask_mma<D>(m, s, tbase, lane, err);
    } else if (warp >= K3_EPI0 / 32) {
        TopK<KM> tk;
        mask_epilogue<D, KM, NW>(m, s, Kidx_bh, qmin_blk, tbase, warp, lane, et, qpos, tk, err);
        mask_merge<KM, NW>(m, s, tk, reinterpret_cast<unsigned long long*>(m.sK), row, et / TILE, qv, qrow,
                           nullptr, nullptr, mv);
        uint8_t* Mrow = M + ((size_t)bh * s.nQB + qb) * s.nKB;
        for (int i = et; i < s.nKB; i += NE) Mrow[i] = m.flags[i];
        // phase B's schedule: the active key blocks in ascending order
        if (et < NEPI) {
            const int w = et >> 5;
            int total = 0;
            for (int b0 = 0; b0 < s.nKB; b0 += NEPI) {
                const int kb = b0 + et;
                const bool v = kb < s.nKB && m.flags[kb];
                const uint32_t bal = __ballot_sync(0xffffffffu, v);
                if (lane == 0) misc[w] = __popc(bal);
                epi_bar();
                int before = 0, all = 0;
                for (int i = 0; i < NEPI / 32; ++i) {
                    before += i < w ? misc[i] : 0;
                    all += misc[i];
                }
                if (v) sched_b[total + before + __popc(bal & ((1u << lane) - 1))] = sched_entry(s, bd, bh, qb, kb, kb);
                total += all;
                epi_bar();
            }
            if (et == 0) misc[9] = total;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    f.T = misc[9];

    // ---- phase B: the forward over the active key blocks
    if (warp == 0) {
        fwd_produce<D>(f, &tmK, &tmV, s, bh, lane, 0, nullptr, err);
    } else if (warp == 1) {
        fwd_mma_s<D>(f, s, tbase, lane, nullptr, err);
    } else if (warp == 2) {
        fwd_mma_pv<D>(f, s, tbase, lane, split, err);
    } else {
        if (et < TILE) {
            // τ from the merged top-k (k1_tau_solve's solve on the same values)
            const float tq = qv ? ref_tau<KM>(mv, s.k, s.alpha) : 0.0f;
            if (qv) tau[qrow] = tq;
            tau_s[row] = tq;
        }
        asm volatile("bar.sync 2, %0;" ::"n"(NE) : "memory");
        fwd_epilogue<D, TO, PINV, NW>(f, s, Kidx_bh, qmin_blk, tbase, warp, lane, et, bh, qb, qpos, tau_s[row],
                                      O, O32, &tmO32, &tmO, rownorm, split, err);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
}

// ===========================================================================
// K4 dQ: query-major over the CSR list.  S = Q·K^T, dP = dO·V^T into TMEM;
// the epilogue (warpgroup h owns key columns [64h, 64h+64)) writes dS as a
// bf16 hi/lo pair into TMEM; dQ += dS·K with dS as the TMEM A operand and
// the K tile as the MN-major B operand.  TMEM: S 0-127, dP 128-255,
// dQ 256-383, dS hi 384-447, dS lo 448-511.  K and V have two stages each;
// V is released after dP, K after dQ.
// ===========================================================================
template <int D, typename TO, int PE2, int SV>
__global__ void __launch_bounds__(DQ_THREADS, 1)
k4_dq(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
      const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO, Shape s,
      const int32_t* __restrict__ Qidx, const int32_t* __restrict__ Kidx, Bounds bd,
      const float* __restrict__ tau, const float* __restrict__ invNv, const float* __restrict__ Dqv,
      const int32_t* __restrict__ ptr, const int32_t* __restrict__ idx, TO* __restrict__ dQ, int split,
      int* err) {
    // K is held from S(j) until dQ(j) (a tile later), V only until dP(j):
    // three K stages, SV V stages (two when shared memory allows).
    constexpr int SK = 3;
    constexpr int TB = D * TILE * 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = align1024(smem_raw, err);
    uint8_t* sQ = base;
    uint8_t* sdO = base + TB;
    uint8_t* sK = base + 2 * TB;              // SK stages
    uint8_t* sV = sK + SK * TB;               // SV stages
    uint64_t* bars = reinterpret_cast<uint64_t*>(sV + SV * TB);
    uint64_t* q_full = bars;
    uint64_t* k_full = bars + 1;
    uint64_t* k_empty = k_full + SK;
    uint64_t* v_full = k_empty + SK;
    uint64_t* v_empty = v_full + SV;
    uint64_t* sd_full = v_empty + SV;
    uint64_t* sd_free = sd_full + 1;
    uint64_t* ds_full = sd_free + 1;
    uint64_t* ds_free = ds_full + 1;
    uint64_t* dq_full = ds_free + 1;
    uint64_t* fixed = dq_full + 1;            // K/V of a tile-load-zeroing tile fixed
    uint64_t* drain = fixed + 1;              // [2] exit-time MMA drains (after a timed-out wait)
    uint32_t* holder = reinterpret_cast<uint32_t*>(bars + 24);
    int* qidx_blk = reinterpret_cast<int*>(holder + 4);
    uint32_t* sched = reinterpret_cast<uint32_t*>(qidx_blk + TILE);   // [T]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int2 bq = grid_order(s.BH, s.nQB, s.causal != 0);
    const int bh = bq.x, qb = bq.y;
    const int32_t* Kidx_bh = Kidx + (size_t)bh * s.NK;
    const int32_t* list = idx + (size_t)bh * s.nQB * s.nKB;
    const int e0 = ptr[(size_t)bh * (s.nQB + 1) + qb];
    const int T = ptr[(size_t)bh * (s.nQB + 1) + qb + 1] - e0;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < SK; ++i) { mbar_init(&k_full[i], 1); mbar_init(&k_empty[i], 1); }
        for (int i = 0; i < SV; ++i) { mbar_init(&v_full[i], 1); mbar_init(&v_empty[i], 1); }
        mbar_init(sd_full, 1);
        mbar_init(sd_free, DQ_NE / 32);
        mbar_init(ds_full, DQ_NE / 32);
        mbar_init(ds_free, 1);
        mbar_init(dq_full, 1);
        mbar_init(fixed, 8);
        mbar_init(&drain[0], 1);
        mbar_init(&drain[1], 1);
        fence_barrier_init();
        if (T > 0) {
            // Q, dO and the first K/V tiles do not depend on the schedule
            // built below: issue them now so their latency hides the set-up
            const int kb0 = list[e0];
            mbar_expect_tx(q_full, 2 * TB);
            mbar_expect_tx(&k_full[0], TB);
            mbar_expect_tx(&v_full[0], TB);
            for (int bx = 0; bx < D / BOX; ++bx) {
                tma_load_3d(sQ + bx * BOX_BYTES, &tmQ, q_full, bx * BOX, qb * TILE, bh);
                tma_load_3d(sdO + bx * BOX_BYTES, &tmdO, q_full, bx * BOX, qb * TILE, bh);
                tma_load_3d(sK + bx * BOX_BYTES, &tmK, &k_full[0], bx * BOX, kb0 * TILE, bh);
                tma_load_3d(sV + bx * BOX_BYTES, &tmV, &v_full[0], bx * BOX, kb0 * TILE, bh);
            }
        }
    }
    if (warp == 1) { tmem_alloc(holder, 512); tmem_relinquish(); }
    if (threadIdx.x >= DQ_EPI0) {
        const int r = threadIdx.x - DQ_EPI0;
        const int q = qb * TILE + r;
        if (r < TILE) qidx_blk[r] = (q < s.NQ && s.causal) ? Qidx[(size_t)bh * s.NQ + q] : INT_MAX;
        if (r < NEPI) sched_from_list(sched, list + e0, T, s, bd, bh, qb, false, r);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *holder;
    constexpr uint32_t tS = 0, tP = 128, tQ = 256, tDh = 384, tDl = 448;
    const int qmin_blk = s.causal ? bd.qmin[bh * s.nQB + qb] : INT_MIN;

    if (warp == 0) {
        if (lane == 0 && T > 0) {
            for (int j = 1; j < T; ++j) {   // Q, dO and tile 0 were issued at set-up
                const int kb = (int)(sched[j] & SCHED_IDX);
                const int st = j % SK;
                mbar_wait(&k_empty[st], ((j / SK) & 1) ^ 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                mbar_expect_tx(&k_full[st], TB);
                for (int bx = 0; bx < D / BOX; ++bx)
                    tma_load_3d(sK + st * TB + bx * BOX_BYTES, &tmK, &k_full[st], bx * BOX, kb * TILE, bh);
            }
        } else if (lane == 1 && T > 0) {
            // V (freed after dP) on its own thread, ahead of K (freed after dQ)
            for (int j = 1; j < T; ++j) {
                const int kb = (int)(sched[j] & SCHED_IDX);
                const int st = j % SV;
                mbar_wait(&v_empty[st], ((j / SV) & 1) ^ 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                mbar_expect_tx(&v_full[st], TB);
                for (int bx = 0; bx < D / BOX; ++bx)
                    tma_load_3d(sV + st * TB + bx * BOX_BYTES, &tmV, &v_full[st], bx * BOX, kb * TILE, bh);
            }
        }
        __syncwarp();
        if (lane == 0 && T > 0 && error_set(err)) {   // a wait gave up: let this CTA's loads land
            mbar_drain(q_full, 0);
            drain_ring(k_full, SK, T);
            drain_ring(v_full, SV, T);
        }
    } else if (warp == 1) {
        // S = Q·K^T and dP = dO·V^T issuer.  dQ comes from warp 2, so the
        // tensor pipe always has the other warp's work while one waits.
        constexpr uint32_t idS = idesc_bf16(128, 128, 0, 0);
        if (T > 0) mbar_wait(q_full, 0, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
        const uint64_t dQd = kdesc(sQ, 0), dOd = kdesc(sdO, 0);
        int nfix = 0;
        for (int j = 0; j < T; ++j) {
            const uint32_t e = sched[j];
            const int kb = (int)(e & SCHED_IDX);
            const bool fix = (e & SCHED_FIX) != 0;
            const int st = j % SK, sv = j % SV;
            uint8_t* kt = sK + st * TB;
            uint8_t* vt = sV + sv * TB;
            mbar_wait(&k_full[st], (j / SK) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            mbar_wait(&v_full[sv], (j / SV) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            if (fix)      // the epilogue warps zero K and V of this tile
                mbar_wait(fixed, (nfix++) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            __syncwarp();
            mbar_wait(sd_free, (j & 1) ^ 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            tc_fence_after();
            if (lane == 0) {
                const uint64_t dK = kdesc(kt, 0), dV = kdesc(vt, 0);
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    mma_bf16_ss(tbase + tS, kdesc_step(dQd, kk), kdesc_step(dK, kk), idS, kk > 0);
                    mma_bf16_ss(tbase + tP, kdesc_step(dOd, kk), kdesc_step(dV, kk), idS, kk > 0);
                }
                mma_commit(sd_full);
                mma_commit(&v_empty[sv]);
            }
            __syncwarp();
        }
        if (lane == 0 && error_set(err)) {   // a wait gave up: let this warp's MMAs finish
            mma_commit(&drain[0]);
            mbar_drain(&drain[0], 0);
        }
        __syncwarp();
    } else if (warp == 2) {
        // dQ += dS·K issuer (in tile order: a deterministic sum)
        constexpr uint32_t idQ = idesc_bf16(128, D, 0, 1);
        for (int i = 0; i < T; ++i) {
            const int st = i % SK;
            const uint8_t* kt = sK + st * TB;
            mbar_wait(ds_full, i & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            tc_fence_after();
            if (lane == 0) {
                const uint64_t dK = mndesc(kt, 0);
#pragma unroll
                for (int kk = 0; kk < TILE / 16; ++kk)
                    mma_bf16_ts(tbase + tQ, tbase + tDh + kk * 8, mndesc_step(dK, kk), idQ, (i > 0 || kk > 0));
                if (split) {
#pragma unroll
                    for (int kk = 0; kk < TILE / 16; ++kk)
                        mma_bf16_ts(tbase + tQ, tbase + tDl + kk * 8, mndesc_step(dK, kk), idQ, 1);
                }
                mma_commit(ds_free);
                mma_commit(&k_empty[st]);
            }
            __syncwarp();
        }
        if (lane == 0) mma_commit(dq_full);
        if (lane == 0 && error_set(err)) {   // a wait gave up: let this warp's MMAs finish
            mma_commit(&drain[1]);
            mbar_drain(&drain[1], 0);
        }
        __syncwarp();
    } else {
        // DQ_NW warpgroups; warpgroup h owns the 32-column chunk h of every
        // tile (D = 128: four chunks).  S and dP are released as soon as they
        // are in registers, so the next tile's S/dP overlaps this gradient.
        const int row = (warp & 3) * 32 + lane;
        const int et = threadIdx.x - DQ_EPI0;
        const int h = et / TILE;
        const int q = qb * TILE + row;
        const bool qv = q < s.NQ;
        const size_t qrow = (size_t)bh * s.NQ + (qv ? q : 0);
        const int qpos = !qv ? INT_MIN : (s.causal ? Qidx[qrow] : INT_MAX);
        const float tq = qv ? tau[qrow] : 0.0f;
        const float invN = qv ? invNv[qrow] : 0.0f;
        const float Dq = qv ? Dqv[qrow] : 0.0f;
        const uint32_t tl = tmem_lane_base(tbase, warp);
        // packed path: u = min(raw·(α-1)·scale - τ, (α-1)·10 - τ); the clamp
        // at -10 can only meet u <= 0, where the gradient is 0
        constexpr bool kPacked = PE2 == 1 || PE2 == 3 || PE2 == 5;
        const bool packed_row = kPacked && qv && __fmaf_rn(s.am1, -10.0f, -tq) <= 0.0f;
        const float2 c1 = make_float2(__fmul_rn(s.am1, s.scale), __fmul_rn(s.am1, s.scale));
        const float2 mtau = make_float2(-tq, -tq), mD = make_float2(-Dq, -Dq), iN = make_float2(invN, invN);
        const float uhi = __fmaf_rn(s.am1, 10.0f, -tq);
        for (int j = 0; j < T; ++j) {
            const uint32_t e = sched[j];
            const int kb = (int)(e & SCHED_IDX);
            const bool all = qv && (e & SCHED_ALL) != 0;
            if ((e & SCHED_FIX) && et < 8 * 32) {
                // the reference's tile-load zeroing of K and V, by eight
                // epilogue warps (32 rows each of K or V); S/dP waits for it
                const int ew = et >> 5;
                uint8_t* tile;
                if (ew < 4) {
                    mbar_wait(&k_full[j % SK], (j / SK) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                    tile = sK + (j % SK) * TB;
                } else {
                    mbar_wait(&v_full[j % SV], (j / SV) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                    tile = sV + (j % SV) * TB;
                }
                fix_tile<D, 1>(tile, qidx_blk, qmin_blk, Kidx_bh, kb, s.NK, lane, 32 * (ew & 3));
                fence_async_smem();
                epi_arrive(fixed);
            }
            mbar_wait(sd_full, j & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            tc_fence_after();
            uint32_t rs[32], rp[32];
            tmem_ld32(tl + tS + h * 32, rs);
            tmem_ld32(tl + tP + h * 32, rp);
            tmem_ld_wait();
            tc_fence_before();
            epi_arrive(sd_free);
            uint32_t hi[16], lo[16];
            if (all && packed_row) {
#pragma unroll
                for (int m = 0; m < 16; ++m) {
                    float2 u = __ffma2_rn(make_float2(__uint_as_float(rs[2 * m]), __uint_as_float(rs[2 * m + 1])),
                                          c1, mtau);
                    u.x = fminf(u.x, uhi);
                    u.y = fminf(u.y, uhi);
                    const float2 t = __fadd2_rn(make_float2(__uint_as_float(rp[2 * m]), __uint_as_float(rp[2 * m + 1])),
                                                mD);
                    float2 g;
                    if constexpr (PE2 == 5) g = t;
                    else if constexpr (PE2 == 1) g = __fmul2_rn(u, t);
                    else g = __fmul2_rn(__fmul2_rn(__fmul2_rn(u, u), u), t);
                    g = __fmul2_rn(g, iN);
                    // u <= EPS or a non-finite product -> 0 (reference :481-507)
                    g.x = (u.x > ASA_EPS && fabsf(g.x) < __int_as_float(0x7f800000)) ? g.x : 0.0f;
                    g.y = (u.y > ASA_EPS && fabsf(g.y) < __int_as_float(0x7f800000)) ? g.y : 0.0f;
                    split_pair(g, hi[m], lo[m]);
                }
            } else {
                const uint32_t vis = all ? 0xffffffffu
                                         : (qv ? vis_mask32(Kidx_bh, kb * TILE + h * 32, s.NK, s.causal, qpos) : 0u);
                float g[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const bool v = (vis >> i) & 1u;
                    const float u = __fmaf_rn(s.am1, clamp_score(__uint_as_float(rs[i]), s.scale), -tq);
                    g[i] = v ? grad_pk<PE2>(u, s.pe2.e, __uint_as_float(rp[i]), Dq, invN) : 0.0f;
                }
                split_pack(g, hi, lo);
            }
            mbar_wait(ds_free, (j & 1) ^ 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            tc_fence_after();
            tmem_st16(tl + tDh + h * 16, hi);
            if (split) tmem_st16(tl + tDl + h * 16, lo);
            tmem_st_wait();
            tc_fence_before();
            epi_arrive(ds_full);
        }
        mbar_wait(dq_full, 0, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
        tc_fence_after();
        // every MMA is done: the Q/dO/K/V tiles are free for the store staging
        float* stage = reinterpret_cast<float*>(sQ) + (et >> 5) * (32 * 33);
        const int q0 = qb * TILE + (warp & 3) * 32;
        const int nrows = min(32, s.NQ - q0);
        const size_t row0 = (size_t)bh * s.NQ + q0;
#pragma unroll 1
        for (int c = h; c < D / 32; c += DQ_NW) {
            uint32_t r[32];
            tmem_ld32(tl + tQ + c * 32, r);
            tmem_ld_wait();
            if (nrows <= 0) continue;
            float o[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                float v = T > 0 ? __uint_as_float(r[i]) * s.scale : 0.0f;
                o[i] = isfinite(v) ? v : 0.0f;
            }
            warp_store_rows<TO>(dQ + row0 * D, D, nrows, c * 32, o, stage, lane);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
}

// ===========================================================================
// K4 dK/dV: key-major over the transposed list.  S^T = K·Q^T and
// dP^T = V·dO^T land in TMEM columns 0-127 and 128-255; the epilogue
// (thread = key row; warpgroup h owns queries [32h, 32h+32)) reads 16
// queries of both at a time and writes P^T/n and dS^T back over those same
// 16 columns as bf16 hi/lo pairs (8 columns each), so no thread overwrites
// data another still reads.
// Then dV += (P^T/n)·dO and dK += dS^T·Q with the pairs as TMEM A operands
// (dV 256-383, dK 384-511).  Q and dO have two stages.
// ===========================================================================
// TMEM column of k-step kk (queries 16kk .. 16kk+15) of the hi (or lo)
// half: each 16-query group's 16 fp32 columns become 8 hi + 8 lo columns.
__device__ __forceinline__ uint32_t pair_col(int kk, bool lo) {
    return (uint32_t)(kk * 16 + (lo ? 8 : 0));
}

template <int D, typename TO, int PINV, int PE2>
__global__ void __launch_bounds__(DKV_THREADS, 1)
k4_dkdv(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO, Shape s,
        const int32_t* __restrict__ Qidx, const int32_t* __restrict__ Kidx, Bounds bd,
        const float* __restrict__ tau, const float* __restrict__ invNv, const float* __restrict__ Dqv,
        const int32_t* __restrict__ cptr, const int32_t* __restrict__ cidx, TO* __restrict__ dK,
        TO* __restrict__ dV, int split, int* err) {
    // Each 128-query tile is handled as two 64-query halves with their own
    // TMEM buffers (S^T 64 columns + dP^T 64 columns each, P^T / dS^T written
    // back over them), so the tensor pipe computes one half's S^T/dP^T while
    // the epilogue works on the other and the dV/dK MMAs drain a third.
    constexpr int SQ = 2;                     // Q / dO stages
    constexpr int TB = D * TILE * 2;
    constexpr int HQ = TILE / 2;              // queries per half
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = align1024(smem_raw, err);
    uint8_t* sK = base;
    uint8_t* sV = base + TB;
    uint8_t* sQ = base + 2 * TB;              // SQ stages
    uint8_t* sdO = sQ + SQ * TB;              // SQ stages
    uint64_t* bars = reinterpret_cast<uint64_t*>(sdO + SQ * TB);
    uint64_t* kv_full = bars;
    uint64_t* q_full = bars + 1;              // [SQ]
    uint64_t* q_empty = q_full + SQ;          // [SQ]
    uint64_t* sd_full = q_empty + SQ;         // [2] per half buffer
    uint64_t* pd_full = sd_full + 2;          // [2]
    uint64_t* pd_free = pd_full + 2;          // [2]
    uint64_t* out_full = pd_free + 2;
    uint64_t* kv_ready = out_full + 1;        // pristine K/V and block positions in place
    uint64_t* fixed = kv_ready + 1;           // ... and zeroed by the epilogue warps
    uint64_t* drain = fixed + 1;              // [2] exit-time MMA drains (after a timed-out wait)
    uint32_t* holder = reinterpret_cast<uint32_t*>(bars + 16);
    // per query of the current (and next) block: query pairs as float4
    // (-τ, -τ', max(lo, 0), max(lo', 0)) and (hi, hi', 1/n, 1/n') with lo/hi
    // the u bounds of the score clamp, then -D and the position per query
    float* qinfo = reinterpret_cast<float*>(holder + 4);     // [2][6][128]
    int* qidx_blk = reinterpret_cast<int*>(qinfo + 2 * 6 * TILE); // [128] for the tile-load fix
    uint32_t* sched = reinterpret_cast<uint32_t*>(qidx_blk + TILE);   // [T]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int2 bk = grid_order(s.BH, s.nKB, false);   // low key blocks (seen by most queries) first
    const int bh = bk.x, kb = bk.y;
    const int32_t* Kidx_bh = Kidx + (size_t)bh * s.NK;
    const int32_t* Qidx_bh = Qidx + (size_t)bh * s.NQ;
    const int32_t* list = cidx + (size_t)bh * s.nKB * s.nQB;
    const int e0 = cptr[(size_t)bh * (s.nKB + 1) + kb];
    const int T = cptr[(size_t)bh * (s.nKB + 1) + kb + 1] - e0;

    if (threadIdx.x == 0) {
        mbar_init(kv_full, 1);
        for (int i = 0; i < SQ; ++i) { mbar_init(&q_full[i], 1); mbar_init(&q_empty[i], 1); }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sd_full[i], 1); mbar_init(&pd_full[i], DKV_NE / 32); mbar_init(&pd_free[i], 1);
        }
        mbar_init(out_full, 1);
        mbar_init(kv_ready, 1);
        mbar_init(fixed, 8);
        mbar_init(&drain[0], 1);
        mbar_init(&drain[1], 1);
        fence_barrier_init();
        if (T > 0) {
            // the first Q/dO tile does not depend on the schedule built below
            const int qb0 = list[e0];
            mbar_expect_tx(&q_full[0], 2 * TB);
            for (int bx = 0; bx < D / BOX; ++bx) {
                tma_load_3d(sQ + bx * BOX_BYTES, &tmQ, &q_full[0], bx * BOX, qb0 * TILE, bh);
                tma_load_3d(sdO + bx * BOX_BYTES, &tmdO, &q_full[0], bx * BOX, qb0 * TILE, bh);
            }
        }
    }
    if (warp == 1) { tmem_alloc(holder, 512); tmem_relinquish(); }
    if (threadIdx.x >= DKV_EPI0 && threadIdx.x < DKV_EPI0 + NEPI)
        sched_from_list(sched, list + e0, T, s, bd, bh, kb, true, threadIdx.x - DKV_EPI0);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *holder;
    // half buffer hb: S^T at 128*hb, dP^T at 128*hb + 64; then dV, dK
    constexpr uint32_t tV = 256, tK = 256 + D;

    if (warp == 0) {
        if (lane == 0 && T > 0) {
            for (int i = 1; i < T; ++i) {   // tile 0 was issued at set-up
                const int qb = (int)(sched[i] & SCHED_IDX);
                const int st = i % SQ;
                mbar_wait(&q_empty[st], ((i / SQ) & 1) ^ 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                mbar_expect_tx(&q_full[st], 2 * TB);
                for (int bx = 0; bx < D / BOX; ++bx) {
                    tma_load_3d(sQ + st * TB + bx * BOX_BYTES, &tmQ, &q_full[st], bx * BOX, qb * TILE, bh);
                    tma_load_3d(sdO + st * TB + bx * BOX_BYTES, &tmdO, &q_full[st], bx * BOX, qb * TILE, bh);
                }
            }
        }
        if (lane == 0 && error_set(err)) drain_ring(q_full, SQ, T);   // a wait gave up: let loads land
    } else if (warp == 1) {
        // S^T = K·Q^T and dP^T = V·dO^T per half (N = 64 queries)
        constexpr uint32_t idS = idesc_bf16(128, HQ, 0, 0);
        int loads = 0, nfix = 0;
        bool dirty = true;   // K/V not loaded yet
        for (int i = 0; i < T; ++i) {
            const uint32_t e = sched[i];
            const int qb = (int)(e & SCHED_IDX);
            const bool fix = (e & SCHED_FIX) != 0;
            const int st = i % SQ;
            if (dirty || fix) {
                // (re)load pristine K/V once the previous tile's S/dP MMAs are done
                if (i > 0) {
                    mbar_wait(&sd_full[0], (i - 1) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                    mbar_wait(&sd_full[1], (i - 1) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                }
                if (lane == 0) {
                    mbar_expect_tx(kv_full, 2 * TB);
                    for (int bx = 0; bx < D / BOX; ++bx) {
                        tma_load_3d(sK + bx * BOX_BYTES, &tmK, kv_full, bx * BOX, kb * TILE, bh);
                        tma_load_3d(sV + bx * BOX_BYTES, &tmV, kv_full, bx * BOX, kb * TILE, bh);
                    }
                }
                mbar_wait(kv_full, loads & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                ++loads;
                if (fix) {
                    for (int r = lane; r < TILE; r += 32) {
                        const int q = qb * TILE + r;
                        qidx_blk[r] = q < s.NQ ? Qidx_bh[q] : INT_MAX;
                    }
                    __syncwarp();
                    // eight epilogue warps zero K and V (32 rows each) while
                    // they would otherwise wait for this tile's S^T/dP^T
                    if (lane == 0) mbar_arrive(kv_ready);
                    mbar_wait(fixed, nfix & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                    ++nfix;
                }
                dirty = fix;
            }
            __syncwarp();
            mbar_wait(&q_full[st], (i / SQ) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            const uint8_t* qt = sQ + st * TB;
            const uint8_t* ot = sdO + st * TB;
            const uint64_t dKd = kdesc(sK, 0), dVd = kdesc(sV, 0);
#pragma unroll 1
            for (int hb = 0; hb < 2; ++hb) {
                mbar_wait(&pd_free[hb], (i & 1) ^ 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                tc_fence_after();
                if (lane == 0) {
                    const uint64_t dQh = kdesc(qt + hb * HQ * 128, 0), dOh = kdesc(ot + hb * HQ * 128, 0);
#pragma unroll
                    for (int kk = 0; kk < D / 16; ++kk) {
                        mma_bf16_ss(tbase + 128 * hb, kdesc_step(dKd, kk), kdesc_step(dQh, kk), idS, kk > 0);
                        mma_bf16_ss(tbase + 128 * hb + 64, kdesc_step(dVd, kk), kdesc_step(dOh, kk), idS, kk > 0);
                    }
                    mma_commit(&sd_full[hb]);
                }
                __syncwarp();
            }
        }
        if (lane == 0 && error_set(err)) {   // a wait gave up: let this warp's loads and MMAs finish
            if (loads > 0) mbar_drain(kv_full, (uint32_t)(loads - 1) & 1u);
            mma_commit(&drain[0]);
            mbar_drain(&drain[0], 0);
        }
        __syncwarp();
    } else if (warp == 2) {
        // dV += P^T·dO and dK += dS^T·Q per half (K = the half's 64 queries),
        // in tile order: deterministic sums
        constexpr uint32_t idO = idesc_bf16(128, D, 0, 1);
        for (int i = 0; i < T; ++i) {
            const int st = i % SQ;
            const uint8_t* qt = sQ + st * TB;
            const uint8_t* ot = sdO + st * TB;
            const uint64_t dOd = mndesc(ot, 0), dQd = mndesc(qt, 0);
#pragma unroll 1
            for (int hb = 0; hb < 2; ++hb) {
                mbar_wait(&pd_full[hb], i & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t cS = tbase + 128 * hb, cP = cS + 64;
#pragma unroll
                    for (int k4 = 0; k4 < HQ / 16; ++k4) {
                        const int kk = hb * (HQ / 16) + k4;
                        const bool acc = i > 0 || kk > 0;
                        mma_bf16_ts(tbase + tV, cS + pair_col(k4, false), mndesc_step(dOd, kk), idO, acc);
                        mma_bf16_ts(tbase + tK, cP + pair_col(k4, false), mndesc_step(dQd, kk), idO, acc);
                    }
                    if (split) {
#pragma unroll
                        for (int k4 = 0; k4 < HQ / 16; ++k4) {
                            const int kk = hb * (HQ / 16) + k4;
                            mma_bf16_ts(tbase + tV, cS + pair_col(k4, true), mndesc_step(dOd, kk), idO, 1);
                            mma_bf16_ts(tbase + tK, cP + pair_col(k4, true), mndesc_step(dQd, kk), idO, 1);
                        }
                    }
                    mma_commit(&pd_free[hb]);
                    if (hb == 1) mma_commit(&q_empty[st]);
                }
                __syncwarp();
            }
        }
        if (lane == 0) mma_commit(out_full);
        if (lane == 0 && error_set(err)) {   // a wait gave up: let this warp's MMAs finish
            mma_commit(&drain[1]);
            mbar_drain(&drain[1], 0);
        }
        __syncwarp();
    } else {
        // DKV_NW warpgroups; in each half warpgroup h owns one 16-query group
        const int row = (warp & 3) * 32 + lane;
        const int et = threadIdx.x - DKV_EPI0;
        const int h = et / TILE;
        const int kn = kb * TILE + row;
        const bool kv = kn < s.NK;
        const size_t krow = (size_t)bh * s.NK + (kv ? kn : 0);
        const int kpos = !kv ? INT_MAX : (s.causal ? Kidx_bh[kn] : INT_MIN);
        const uint32_t tl = tmem_lane_base(tbase, warp);
        constexpr bool kPacked = (PINV == 1 || PINV == 2 || PINV == 4) && (PE2 == 1 || PE2 == 3 || PE2 == 5);
        const float2 c1 = make_float2(__fmul_rn(s.am1, s.scale), __fmul_rn(s.am1, s.scale));
        // Query-block metadata of tile i lives in qinfo[i & 1]; it is fetched
        // one tile ahead so its global loads overlap the previous tile.
        auto fetch = [&](int i, float* dst) {
            const int qb = (int)(sched[i] & SCHED_IDX);
            const int q = qb * TILE + et;
            const bool ok = q < s.NQ;
            const size_t r = (size_t)bh * s.NQ + (ok ? q : 0);
            const float tq = ok ? tau[r] : 0.0f;
            const int pq = (et >> 1) * 4 + (et & 1);
            dst[pq] = -tq;
            dst[pq + 2] = fmaxf(__fmaf_rn(s.am1, -10.0f, -tq), 0.0f);
            dst[256 + pq] = __fmaf_rn(s.am1, 10.0f, -tq);
            dst[256 + pq + 2] = ok ? invNv[r] : 0.0f;
            dst[512 + et] = ok ? -Dqv[r] : 0.0f;
            dst[640 + et] = __int_as_float(ok ? (s.causal ? Qidx_bh[q] : INT_MAX) : INT_MIN);
        };
        if (T > 0 && et < TILE) fetch(0, qinfo);
        int nfix = 0;
        for (int i = 0; i < T; ++i) {
            const uint32_t e = sched[i];
            asm volatile("bar.sync 2, %0;" ::"n"(DKV_NE) : "memory");   // qinfo[i&1] written; tile i-1 done
            if (i + 1 < T && et < TILE) fetch(i + 1, qinfo + ((i + 1) & 1) * 6 * TILE);
            const float* qi = qinfo + (i & 1) * 6 * TILE;
            if ((e & SCHED_FIX) && et < 8 * 32) {
                const int ew = et >> 5;
                mbar_wait(kv_ready, nfix & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                const int qbf = (int)(e & SCHED_IDX);
                fix_tile<D, 1>(ew < 4 ? sK : sV, qidx_blk, bd.qmin[bh * s.nQB + qbf], Kidx_bh, kb, s.NK, lane,
                               32 * (ew & 3));
                fence_async_smem();
                epi_arrive(fixed);
            }
            if (e & SCHED_FIX) ++nfix;
            const bool all = kv && (e & SCHED_ALL) != 0;
#pragma unroll 1
            for (int hb = 0; hb < 2; ++hb) {
                const int gq = hb * 4 + h;            // 16-query group of the tile
                const uint32_t cS = 128 * hb, cP = cS + 64;
                mbar_wait(&sd_full[hb], i & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                tc_fence_after();
                uint32_t rs[16], rp[16];
                tmem_ld16(tl + cS + h * 16, rs);
                tmem_ld16(tl + cP + h * 16, rp);
                tmem_ld_wait();
                uint32_t ph[8], pl[8], gh[8], gl[8];
                if (kPacked && all) {
#pragma unroll
                    for (int m = 0; m < 8; ++m) {
                        const int qq = gq * 16 + 2 * m;
                        // pair of queries: (-τ, -τ', max(lo,0), max(lo',0)), (hi, hi', 1/n, 1/n')
                        const float4 qa = *reinterpret_cast<const float4*>(qi + (qq >> 1) * 4);
                        const float4 qb4 = *reinterpret_cast<const float4*>(qi + 256 + (qq >> 1) * 4);
                        const float2 nD = *reinterpret_cast<const float2*>(qi + 512 + qq);
                        const float2 iN = make_float2(qb4.z, qb4.w);
                        float2 u = __ffma2_rn(make_float2(__uint_as_float(rs[2 * m]), __uint_as_float(rs[2 * m + 1])),
                                              c1, make_float2(qa.x, qa.y));
                        // clamp to [max(lo, 0), hi]: below 0 both the weight and the
                        // gradient are 0, so the floor at 0 also gives max(u, 0)
                        u.x = fmaxf(fminf(u.x, qb4.x), qa.z);
                        u.y = fmaxf(fminf(u.y, qb4.y), qa.w);
                        const float2 up = u;
                        float2 pv;
                        if constexpr (PINV == 1) pv = up;
                        else if constexpr (PINV == 2) pv = __fmul2_rn(up, up);
                        else { const float2 q2 = __fmul2_rn(up, up); pv = __fmul2_rn(q2, q2); }
                        pv = __fmul2_rn(pv, iN);
                        const float2 t = __fadd2_rn(make_float2(__uint_as_float(rp[2 * m]), __uint_as_float(rp[2 * m + 1])),
                                                    nD);
                        float2 g;
                        if constexpr (PE2 == 5) g = t;
                        else if constexpr (PE2 == 1) g = __fmul2_rn(u, t);
                        else g = __fmul2_rn(__fmul2_rn(__fmul2_rn(u, u), u), t);
                        g = __fmul2_rn(g, iN);
                        g.x = (u.x > ASA_EPS && fabsf(g.x) < __int_as_float(0x7f800000)) ? g.x : 0.0f;
                        g.y = (u.y > ASA_EPS && fabsf(g.y) < __int_as_float(0x7f800000)) ? g.y : 0.0f;
                        split_pair(pv, ph[m], pl[m]);
                        split_pair(g, gh[m], gl[m]);
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < 16; k += 2) {
                        float pv[2], gv[2];
#pragma unroll
                        for (int t = 0; t < 2; ++t) {
                            const int qq = gq * 16 + k + t;
                            const bool v = all || (kv && kpos <= __float_as_int(qi[640 + qq]));
                            const float u = __fmaf_rn(s.am1, clamp_score(__uint_as_float(rs[k + t]), s.scale),
                                                      qi[(qq >> 1) * 4 + (qq & 1)]);
                            const float iN = qi[256 + (qq >> 1) * 4 + 2 + (qq & 1)];
                            pv[t] = v ? entmax_pk<PINV>(u, s.pinv.e) * iN : 0.0f;
                            gv[t] = v ? grad_pk<PE2>(u, s.pe2.e, __uint_as_float(rp[k + t]), -qi[512 + qq], iN)
                                      : 0.0f;
                        }
                        split_pair(make_float2(pv[0], pv[1]), ph[k >> 1], pl[k >> 1]);
                        split_pair(make_float2(gv[0], gv[1]), gh[k >> 1], gl[k >> 1]);
                    }
                }
                tmem_st8(tl + cS + h * 16, ph);
                if (split) tmem_st8(tl + cS + h * 16 + 8, pl);
                tmem_st8(tl + cP + h * 16, gh);
                if (split) tmem_st8(tl + cP + h * 16 + 8, gl);
                tmem_st_wait();
                tc_fence_before();
                epi_arrive(&pd_full[hb]);
            }
        }
        if (T > 0) {
            mbar_wait(out_full, 0, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            tc_fence_after();
        }
        // every MMA is done: the K/V and Q/dO tiles are free for the store staging
        float* stage = reinterpret_cast<float*>(sK) + (et >> 5) * (32 * 33);
        const int k0 = kb * TILE + (warp & 3) * 32;
        const int nrows = min(32, s.NK - k0);
        const size_t row0 = (size_t)bh * s.NK + k0;
#pragma unroll 1
        for (int part = 0; part < 2; ++part) {
            TO* dst_base = part == 0 ? dV : dK;
            const float mul = part == 0 ? 1.0f : s.scale;
            const uint32_t col0 = part == 0 ? tV : tK;
#pragma unroll 1
            for (int c = h; c < D / 32; c += DKV_NW) {
                uint32_t r[32];
                if (T > 0) {
                    tmem_ld32(tl + col0 + c * 32, r);
                    tmem_ld_wait();
                }
                if (nrows <= 0) continue;
                float o[32];
#pragma unroll
                for (int k = 0; k < 32; ++k) {
                    float v = T > 0 ? __uint_as_float(r[k]) * mul : 0.0f;
                    o[k] = isfinite(v) ? v : 0.0f;
                }
                warp_store_rows<TO>(dst_base + row0 * D, D, nrows, c * 32, o, stage, lane);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
}

// ===========================================================================
// K4 jac: the row statistic of the Jacobian gradient (asa_grad_mode
// ASA_GRAD_JACOBIAN), no counterpart in the reference.  Over the CSR tile
// list: S = Q·K^T and dP = dO·V^T into TMEM (two buffers), and per query
// R = Σ_j w_j dP_j / Σ_j w_j, w = u^{(2-α)/(α-1)} for u > EPS (the weights
// the gradient kernels apply).  R replaces D = O·dO, so dQ and dK/dV then
// compute g = w (dP - R) / n.  Each of the DQ_NW epilogue warpgroups owns
// one 32-key chunk of every tile; the row's partial sums are added in a
// fixed order at the end.
// ===========================================================================
template <int D, int PE2>
__global__ void __launch_bounds__(DQ_THREADS, 1)
k4_jac(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmdO, Shape s,
       const int32_t* __restrict__ Qidx, const int32_t* __restrict__ Kidx, Bounds bd,
       const float* __restrict__ tau, const int32_t* __restrict__ ptr, const int32_t* __restrict__ idx,
       float* __restrict__ Rq, int* err) {
    constexpr int SK = 2, SV = 2;             // K / V stages (both released after S/dP)
    constexpr int NB = 2;                     // S/dP buffer pairs in TMEM
    constexpr int TB = D * TILE * 2;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = align1024(smem_raw, err);
    uint8_t* sQ = base;
    uint8_t* sdO = base + TB;
    uint8_t* sK = base + 2 * TB;              // SK stages
    uint8_t* sV = sK + SK * TB;               // SV stages
    float* red = reinterpret_cast<float*>(sV + SV * TB);    // [2][DQ_NW][128] partial sums
    uint64_t* bars = reinterpret_cast<uint64_t*>(red + 2 * DQ_NW * TILE);
    uint64_t* q_full = bars;
    uint64_t* k_full = bars + 1;
    uint64_t* k_empty = k_full + SK;
    uint64_t* v_full = k_empty + SK;
    uint64_t* v_empty = v_full + SV;
    uint64_t* sd_full = v_empty + SV;         // [NB]
    uint64_t* sd_free = sd_full + NB;         // [NB]
    uint64_t* fixed = sd_free + NB;           // K/V of a tile-load-zeroing tile fixed
    uint64_t* drain = fixed + 1;              // exit-time MMA drain (after a timed-out wait)
    uint32_t* holder = reinterpret_cast<uint32_t*>(bars + 24);
    int* qidx_blk = reinterpret_cast<int*>(holder + 4);
    uint32_t* sched = reinterpret_cast<uint32_t*>(qidx_blk + TILE);   // [T]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int2 bq = grid_order(s.BH, s.nQB, s.causal != 0);
    const int bh = bq.x, qb = bq.y;
    const int32_t* Kidx_bh = Kidx + (size_t)bh * s.NK;
    const int32_t* list = idx + (size_t)bh * s.nQB * s.nKB;
    const int e0 = ptr[(size_t)bh * (s.nQB + 1) + qb];
    const int T = ptr[(size_t)bh * (s.nQB + 1) + qb + 1] - e0;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < SK; ++i) { mbar_init(&k_full[i], 1); mbar_init(&k_empty[i], 1); }
        for (int i = 0; i < SV; ++i) { mbar_init(&v_full[i], 1); mbar_init(&v_empty[i], 1); }
        for (int i = 0; i < NB; ++i) { mbar_init(&sd_full[i], 1); mbar_init(&sd_free[i], DQ_NE / 32); }
        mbar_init(fixed, 8);
        mbar_init(drain, 1);
        fence_barrier_init();
        if (T > 0) {
            mbar_expect_tx(q_full, 2 * TB);
            for (int bx = 0; bx < D / BOX; ++bx) {
                tma_load_3d(sQ + bx * BOX_BYTES, &tmQ, q_full, bx * BOX, qb * TILE, bh);
                tma_load_3d(sdO + bx * BOX_BYTES, &tmdO, q_full, bx * BOX, qb * TILE, bh);
            }
        }
    }
    if (warp == 1) { tmem_alloc(holder, 512); tmem_relinquish(); }
    if (threadIdx.x >= DQ_EPI0) {
        const int r = threadIdx.x - DQ_EPI0;
        const int q = qb * TILE + r;
        if (r < TILE) qidx_blk[r] = (q < s.NQ && s.causal) ? Qidx[(size_t)bh * s.NQ + q] : INT_MAX;
        if (r < NEPI) sched_from_list(sched, list + e0, T, s, bd, bh, qb, false, r);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = *holder;
    const int qmin_blk = s.causal ? bd.qmin[bh * s.nQB + qb] : INT_MIN;

    if (warp == 0) {
        if (lane < 2 && T > 0) {
            // lane 0 streams K, lane 1 streams V
            uint64_t* full = lane == 0 ? k_full : v_full;
            uint64_t* empty = lane == 0 ? k_empty : v_empty;
            uint8_t* ring = lane == 0 ? sK : sV;
            const CUtensorMap* tm = lane == 0 ? &tmK : &tmV;
            for (int j = 0; j < T; ++j) {
                const int kb = (int)(sched[j] & SCHED_IDX);
                const int st = j % 2;
                mbar_wait(&empty[st], ((j / 2) & 1) ^ 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                mbar_expect_tx(&full[st], TB);
                for (int bx = 0; bx < D / BOX; ++bx)
                    tma_load_3d(ring + st * TB + bx * BOX_BYTES, tm, &full[st], bx * BOX, kb * TILE, bh);
            }
        }
        __syncwarp();
        if (lane == 0 && T > 0 && error_set(err)) {   // a wait gave up: let this CTA's loads land
            mbar_drain(q_full, 0);
            drain_ring(k_full, SK, T);
            drain_ring(v_full, SV, T);
        }
    } else if (warp == 1) {
        constexpr uint32_t idS = idesc_bf16(128, 128, 0, 0);
        if (T > 0) mbar_wait(q_full, 0, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
        const uint64_t dQd = kdesc(sQ, 0), dOd = kdesc(sdO, 0);
        int nfix = 0;
        for (int j = 0; j < T; ++j) {
            const int st = j % 2, b = j % NB;
            mbar_wait(&k_full[st], (j / 2) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            mbar_wait(&v_full[st], (j / 2) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            if (sched[j] & SCHED_FIX)      // the epilogue warps zero K and V of this tile
                mbar_wait(fixed, (nfix++) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            __syncwarp();
            mbar_wait(&sd_free[b], ((j / NB) & 1) ^ 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            tc_fence_after();
            if (lane == 0) {
                const uint64_t dK = kdesc(sK + st * TB, 0), dV = kdesc(sV + st * TB, 0);
                const uint32_t cS = tbase + b * 256, cP = cS + 128;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    mma_bf16_ss(cS, kdesc_step(dQd, kk), kdesc_step(dK, kk), idS, kk > 0);
                    mma_bf16_ss(cP, kdesc_step(dOd, kk), kdesc_step(dV, kk), idS, kk > 0);
                }
                mma_commit(&sd_full[b]);
                mma_commit(&k_empty[st]);
                mma_commit(&v_empty[st]);
            }
            __syncwarp();
        }
        if (lane == 0 && error_set(err)) {   // a wait gave up: let this warp's MMAs finish
            mma_commit(drain);
            mbar_drain(drain, 0);
        }
        __syncwarp();
    } else if (warp >= DQ_EPI0 / 32) {
        const int row = (warp & 3) * 32 + lane;
        const int et = threadIdx.x - DQ_EPI0;
        const int h = et / TILE;                  // 32-key chunk of every tile
        const int q = qb * TILE + row;
        const bool qv = q < s.NQ;
        const size_t qrow = (size_t)bh * s.NQ + (qv ? q : 0);
        const int qpos = !qv ? INT_MIN : (s.causal ? Qidx[qrow] : INT_MAX);
        const float tq = qv ? tau[qrow] : 0.0f;
        const uint32_t tl = tmem_lane_base(tbase, warp);
        float A = 0.0f, B = 0.0f;
        // packed path: u = min(raw·(α-1)·scale - τ, (α-1)·10 - τ); the clamp
        // at -10 can only meet u <= 0, where the weight is 0
        constexpr bool kPacked = PE2 == 1 || PE2 == 3 || PE2 == 5;
        const bool packed_row = kPacked && qv && s.scale > 0.0f && __fmaf_rn(s.am1, -10.0f, -tq) <= 0.0f;
        const float c1s = __fmul_rn(s.am1, s.scale);
        const float2 c1 = make_float2(c1s, c1s), mtau = make_float2(-tq, -tq);
        const float uhi = __fmaf_rn(s.am1, 10.0f, -tq);
        for (int j = 0; j < T; ++j) {
            const uint32_t e = sched[j];
            const int kb = (int)(e & SCHED_IDX);
            const int b = j % NB;
            const bool all = qv && (e & SCHED_ALL) != 0;
            if ((e & SCHED_FIX) && et < 8 * 32) {
                // the reference's tile-load zeroing of K and V, by eight
                // epilogue warps (32 rows each of K or V); S/dP waits for it
                const int ew = et >> 5;
                uint8_t* tile;
                if (ew < 4) {
                    mbar_wait(&k_full[j % 2], (j / 2) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                    tile = sK + (j % 2) * TB;
                } else {
                    mbar_wait(&v_full[j % 2], (j / 2) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
                    tile = sV + (j % 2) * TB;
                }
                fix_tile<D, 1>(tile, qidx_blk, qmin_blk, Kidx_bh, kb, s.NK, lane, 32 * (ew & 3));
                fence_async_smem();
                epi_arrive(fixed);
            }
            mbar_wait(&sd_full[b], (j / NB) & 1, s.spins, err, ASA_ERR_DEVICE_TIMEOUT);
            tc_fence_after();
            uint32_t rs[32], rp[32];
            tmem_ld32(tl + b * 256 + h * 32, rs);
            tmem_ld32(tl + b * 256 + 128 + h * 32, rp);
            tmem_ld_wait();
            tc_fence_before();
            epi_arrive(&sd_free[b]);
            const uint32_t vis = all ? 0xffffffffu
                                     : (qv ? vis_mask32(Kidx_bh, kb * TILE + h * 32, s.NK, s.causal, qpos) : 0u);
            if (kPacked && packed_row) {
                float2 a2 = make_float2(0.0f, 0.0f), b2 = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int m = 0; m < 16; ++m) {
                    float2 u = __ffma2_rn(make_float2(__uint_as_float(rs[2 * m]), __uint_as_float(rs[2 * m + 1])),
                                          c1, mtau);
                    u.x = fminf(u.x, uhi);
                    u.y = fminf(u.y, uhi);
                    const bool k0 = ((vis >> (2 * m)) & 1u) && u.x > ASA_EPS;
                    const bool k1v = ((vis >> (2 * m + 1)) & 1u) && u.y > ASA_EPS;
                    float2 w = powk2<PE2>(make_float2(fmaxf(u.x, ASA_EPS), fmaxf(u.y, ASA_EPS)));
                    w.x = k0 ? w.x : 0.0f;
                    w.y = k1v ? w.y : 0.0f;
                    a2 = __ffma2_rn(w, make_float2(__uint_as_float(rp[2 * m]), __uint_as_float(rp[2 * m + 1])), a2);
                    b2 = __fadd2_rn(b2, w);
                }
                A += a2.x + a2.y;
                B += b2.x + b2.y;
                continue;
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                if (!((vis >> i) & 1u)) continue;
                const float u = __fmaf_rn(s.am1, clamp_score(__uint_as_float(rs[i]), s.scale), -tq);
                if (!(u > ASA_EPS)) continue;
                const float w = powk<PE2>(fmaxf(u, ASA_EPS), s.pe2.e);
                if (!isfinite(w)) continue;
                A = fmaf(w, __uint_as_float(rp[i]), A);
                B += w;
            }
        }
        red[h * TILE + row] = A;
        red[(DQ_NW + h) * TILE + row] = B;
        asm volatile("bar.sync 2, %0;" ::"n"(DQ_NE) : "memory");
        if (h == 0 && qv) {
            float a = 0.0f, bs = 0.0f;
#pragma unroll
            for (int g = 0; g < DQ_NW; ++g) {
                a += red[g * TILE + row];
                bs += red[(DQ_NW + g) * TILE + row];
            }
            Rq[qrow] = bs > 0.0f ? a / bs : 0.0f;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
}

// ===========================================================================
// K4 pre: D_q = Σ_t O_t · dO_t (fp32 O, bf16 dO) and 1/(n+EPS).  D/4 lanes
// per row, each reading one float4 of O and four bf16 of dO (16- and 8-byte
// loads: the kernel is HBM-bound); d = 64 puts two rows in a warp.
// ===========================================================================
template <int D>
__global__ void k4_pre(const float* __restrict__ O32, const __nv_bfloat16* __restrict__ dO,
                       const float* __restrict__ rownorm, float* __restrict__ Dq,
                       float* __restrict__ invN, size_t rows) {
    constexpr int LPR = D / 4;                // lanes per row
    constexpr int RPW = 32 / LPR;             // rows per warp
    const int lane = threadIdx.x & 31;
    const int l = lane % LPR;
    const size_t r = ((size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW + lane / LPR;
    float acc = 0.0f;
    if (r < rows) {
        const float4 o = __ldg(reinterpret_cast<const float4*>(O32 + r * D) + l);
        const uint2 g = __ldg(reinterpret_cast<const uint2*>(dO + r * D) + l);
        acc = fmaf(o.x, __uint_as_float(g.x << 16), acc);
        acc = fmaf(o.y, __uint_as_float(g.x & 0xffff0000u), acc);
        acc = fmaf(o.z, __uint_as_float(g.y << 16), acc);
        acc = fmaf(o.w, __uint_as_float(g.y & 0xffff0000u), acc);
    }
#pragma unroll
    for (int off = LPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (l == 0 && r < rows) {
        Dq[r] = acc;
        invN[r] = __fdiv_rn(1.0f, __fadd_rn(rownorm[r], ASA_EPS));   // reference :435
    }
}

// ===========================================================================
// host side
// ===========================================================================
// Looked up once per process; a function-local static's initialisation is
// thread-safe, so concurrent first calls from several host threads are fine.
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            return (PFN_cuTensorMapEncodeTiled_v12000)p;
        return (PFN_cuTensorMapEncodeTiled_v12000) nullptr;
    }();
    return fn;
}

// [BH][N][d] bf16 viewed as a 3-D tensor, boxes of 64 x 128 x 1, 128-byte
// swizzle, zero fill out of bounds.
bool make_map(CUtensorMap* m, const void* ptr, int BH, int N, int d) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)d, (cuuint64_t)N, (cuuint64_t)BH};
    cuuint64_t strides[2] = {(cuuint64_t)d * 2, (cuuint64_t)N * d * 2};
    cuuint32_t box[3] = {BOX, TILE, 1};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box,
                    es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Store map of an output [BH][N][d] (fp32 or bf16): boxes of 32 x 32 x 1,
// swizzled rows (128 B fp32, 64 B bf16) as warp_tma_store stages them.
bool make_store_map(CUtensorMap* m, const void* ptr, int BH, int N, int d, bool f32) {
    auto fn = encode_fn();
    if (!fn) return false;
    const int es = f32 ? 4 : 2;
    cuuint64_t dims[3] = {(cuuint64_t)d, (cuuint64_t)N, (cuuint64_t)BH};
    cuuint64_t strides[2] = {(cuuint64_t)d * es, (cuuint64_t)N * d * es};
    cuuint32_t box[3] = {32, 32, 1};
    cuuint32_t est[3] = {1, 1, 1};
    CUresult r = fn(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                    const_cast<void*>(ptr), dims, strides, box, est, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

size_t bounds_ints(const Shape& s) { return (size_t)2 * s.BH * (s.nQB + s.nKB); }

Bounds bounds_at(const Shape& s, void* ws) {
    int* b = (int*)ws;
    Bounds bd;
    bd.qmin = b;
    bd.qmax = b + (size_t)s.BH * s.nQB;
    bd.kmin = b + (size_t)2 * s.BH * s.nQB;
    bd.kmax = b + (size_t)2 * s.BH * s.nQB + (size_t)s.BH * s.nKB;
    return bd;
}

cudaError_t launch_bounds(const Shape& s, const int32_t* Qidx, const int32_t* Kidx, void* ws,
                          cudaStream_t st) {
    if (!s.causal) return cudaSuccess;
    Bounds bd = bounds_at(s, ws);
    const int blocks = (s.nQB + s.nKB + 7) / 8;
    dim3 grid(blocks, s.BH);
    tc_bounds_kernel<<<grid, 256, 0, st>>>(s, Qidx, Kidx, (int*)bd.qmin, (int*)bd.qmax, (int*)bd.kmin,
                                           (int*)bd.kmax);
    note_launch();
    return cudaGetLastError();
}

template <typename F>
cudaError_t prep(F* f, size_t smem) {
    return cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

// The forward's epilogue width: four warpgroups (one 32-column chunk of each
// tile per thread) when the fused kernel runs the same width, so both forwards
// add a row's weights in the same order.
bool fwd_wide(const Shape& s) { return s.k <= 8; }
constexpr size_t kSmemTailBwd = 16 * 8 + 16 + 2 * 6 * 128 * 4 + 128 * 4;  // + per-query arrays x2

// Whether the current device is sm_100 (per call: a process may use several
// devices; the attribute query is cheap).
bool is_sm100() {
    int dev = 0, major = 0;
    return cudaGetDevice(&dev) == cudaSuccess &&
           cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) == cudaSuccess && major == 10;
}

}  // namespace

#ifndef ASA_TC_PART
#define ASA_TC_PART 0   // 0: everything; 1: τ/mask + sizing, 2: forward, 3: backward prologue + dQ, 4: dK/dV,
                        // 5: fused forward
#endif
#define ASA_PART(n) (ASA_TC_PART == 0 || ASA_TC_PART == (n))

#if ASA_PART(1)
bool tc_supported(const Shape& s) {
    return s.in_dtype == ASA_DTYPE_BF16 && (s.d == 64 || s.d == 128) && s.BM == TILE && s.BN == TILE &&
           s.NK > 0 && s.nKB <= 2048 && is_sm100();   // per-CTA schedules live in shared memory
}

// Forward workspace: [per-block index bounds | per-row top-k scores (k1 -> τ solve)]
size_t topv_offset(const Shape& s) { return (bounds_ints(s) * 4 + 15) & ~size_t(15); }
size_t tc_fwd_workspace(const Shape& s) { return topv_offset(s) + (size_t)s.BH * s.NQ * s.k * 4; }
size_t tc_bwd_workspace(const Shape& s) {
    return ((bounds_ints(s) * 4 + 15) & ~size_t(15)) + (size_t)2 * s.BH * s.NQ * 4;
}

#endif  // part 1

// Exponent classes the kernels are specialised for: (1/(α-1), (2-α)/(α-1))
// kinds (2,1) for α=1.5, (1,5) for α=2, (4,3) for α=1.25; anything else runs
// the generic powf instantiation.
template <int PI, int PE> struct AlphaClass {
    static constexpr int pinv = PI, pe2 = PE;
};
template <typename F>
cudaError_t with_alpha(const Shape& s, F&& f) {
    if (s.pinv.kind == 2 && s.pe2.kind == 1) return f(AlphaClass<2, 1>{});
    if (s.pinv.kind == 1 && s.pe2.kind == 5) return f(AlphaClass<1, 5>{});
    if (s.pinv.kind == 4 && s.pe2.kind == 3) return f(AlphaClass<4, 3>{});
    return f(AlphaClass<0, 0>{});
}
template <typename F>
cudaError_t with_dtype_d(const Shape& s, F&& f) {
    using bf = __nv_bfloat16;
    if (s.out_dtype == ASA_DTYPE_F32) {
        if (s.d == 128) return f(std::integral_constant<int, 128>{}, (float*)nullptr);
        return f(std::integral_constant<int, 64>{}, (float*)nullptr);
    }
    if (s.d == 128) return f(std::integral_constant<int, 128>{}, (bf*)nullptr);
    return f(std::integral_constant<int, 64>{}, (bf*)nullptr);
}

#if ASA_PART(1)
cudaError_t tc_tau_mask(const Shape& s, const void* Q, const void* K, const int32_t* Qidx,
                        const int32_t* Kidx, float* tau, uint8_t* M, void* ws, int* err,
                        cudaStream_t st, float* topv_out, int32_t* topi_out) {
    cudaError_t e = launch_bounds(s, Qidx, Kidx, ws, st);
    if (e != cudaSuccess) return e;
    CUtensorMap mQ, mK;
    if (!make_map(&mQ, Q, s.BH, s.NQ, s.d) || !make_map(&mK, K, s.BH, s.NK, s.d)) return cudaErrorInvalidValue;
    Bounds bd = bounds_at(s, ws);
    dim3 grid(s.BH * s.nQB);
    // the rows' top-k scores (and keys) in order: the caller's buffers, or
    // the workspace when only τ and the mask are wanted
    float* topv = topv_out ? topv_out : (float*)((char*)ws + topv_offset(s));
    const size_t rows = (size_t)s.BH * s.NQ;
    auto go = [&](auto kern, auto solve, int D, int NW) -> cudaError_t {
        const int S = 3;
        // Q, the K stages, chunk copies and bounds, barriers + TMEM holder,
        // positions, counts, the schedule and the flags, alignment slack
        const size_t smem = (size_t)D * TILE * 2 * (1 + S) + (D == 128 ? (NW == 4 ? mask_extra_bytes<128, 4>()
                                                                               : mask_extra_bytes<128, 2>())
                                                                    : (NW == 4 ? mask_extra_bytes<64, 4>()
                                                                               : mask_extra_bytes<64, 2>())) +
                            24 * 8 + 16 + TILE * 4 + 16 * 4 + (size_t)s.nKB * 5 + 64;
        cudaError_t r = prep(kern, smem);
        if (r != cudaSuccess) return r;
        kern<<<grid, 64 + 128 * NW, smem, st>>>(mQ, mK, s, Qidx, Kidx, bd, topv, topi_out, M, err);
        note_launch();
        r = cudaGetLastError();
        if (r != cudaSuccess || !tau) return r;
        solve<<<(unsigned)((rows + 127) / 128), 128, 0, st>>>(topv, tau, rows, s.k, s.alpha);
        note_launch();
        return cudaGetLastError();
    };
    if (s.d == 128) {
        if (s.k <= 8) return go(k1_tau_mask<128, 8, 4>, k1_tau_solve<8>, 128, 4);
        if (s.k <= 16) return go(k1_tau_mask<128, 16, 4>, k1_tau_solve<16>, 128, 4);
        return go(k1_tau_mask<128, 32, 2>, k1_tau_solve<32>, 128, 2);
    }
    if (s.k <= 8) return go(k1_tau_mask<64, 8, 4>, k1_tau_solve<8>, 64, 4);
    if (s.k <= 16) return go(k1_tau_mask<64, 16, 4>, k1_tau_solve<16>, 64, 4);
    return go(k1_tau_mask<64, 32, 2>, k1_tau_solve<32>, 64, 2);
}

// τ and the mask by the exact α-entmax threshold (asa_tau_mode ASA_TAU_EXACT).
cudaError_t tc_exact_tau(const Shape& s, const void* Q, const void* K, const int32_t* Qidx,
                         const int32_t* Kidx, float* tau, uint8_t* M, void* ws, int* err,
                         cudaStream_t st) {
    cudaError_t e = launch_bounds(s, Qidx, Kidx, ws, st);
    if (e != cudaSuccess) return e;
    CUtensorMap mQ, mK;
    if (!make_map(&mQ, Q, s.BH, s.NQ, s.d) || !make_map(&mK, K, s.BH, s.NK, s.d)) return cudaErrorInvalidValue;
    Bounds bd = bounds_at(s, ws);
    dim3 grid(s.BH * s.nQB);
    return with_alpha(s, [&](auto ac) -> cudaError_t {
        constexpr int PI = decltype(ac)::pinv, PE = decltype(ac)::pe2;
        auto go = [&](auto kern, int D) -> cudaError_t {
            // Q + four K stages, partial sums, barriers + TMEM holder, counts,
            // the tile schedule and the mask flags, alignment slack
            const size_t smem = (size_t)D * TILE * 2 * 5 + (size_t)4 * 4 * TILE * 4 + 24 * 8 + 16 + 64 +
                                (size_t)s.nKB * 5 + 64;
            cudaError_t r = prep(kern, smem);
            if (r != cudaSuccess) return r;
            kern<<<grid, 64 + 128 * 4, smem, st>>>(mQ, mK, s, Qidx, Kidx, bd, tau, M, err);
            note_launch();
            return cudaGetLastError();
        };
        if (s.d == 128) return go(k1_exact<128, 4, PI, PE>, 128);
        return go(k1_exact<64, 4, PI, PE>, 64);
    });
}

#endif  // part 1

#if ASA_PART(2)
cudaError_t tc_forward(const Shape& s, const void* Q, const void* K, const void* V, const int32_t* Qidx,
                       const int32_t* Kidx, const float* tau, const int32_t* ptr, const int32_t* idx,
                       void* O, float* O32, float* rownorm, void* ws, int* err, cudaStream_t st) {
    CUtensorMap mQ, mK, mV, mO32, mO;
    if (!make_map(&mQ, Q, s.BH, s.NQ, s.d) || !make_map(&mK, K, s.BH, s.NK, s.d) ||
        !make_map(&mV, V, s.BH, s.NK, s.d) ||
        !make_store_map(&mO, O, s.BH, s.NQ, s.d, s.out_dtype == ASA_DTYPE_F32))
        return cudaErrorInvalidValue;
    if (!O32) mO32 = mO;   // not stored
    else if (!make_store_map(&mO32, O32, s.BH, s.NQ, s.d, true)) return cudaErrorInvalidValue;
    Bounds bd = bounds_at(s, ws);   // filled by tc_tau_mask
    dim3 grid(s.BH * s.nQB);
    const int split = s.split;
    return with_dtype_d(s, [&](auto dtag, auto* out) -> cudaError_t {
        constexpr int D = decltype(dtag)::value;
        using TO = std::remove_pointer_t<decltype(out)>;
        return with_alpha(s, [&](auto ac) -> cudaError_t {
            auto go = [&](auto k, auto nw) -> cudaError_t {
                constexpr int NW = decltype(nw)::value;
                // Q, K and V stages, barriers + TMEM holder, per-row arrays, the schedule
                const size_t smem = (size_t)D * TILE * 2 * 6 + 24 * 8 + 16 + (size_t)(NW + 1) * TILE * 4 + 64 +
                                    (size_t)s.nKB * 4;
                cudaError_t r = prep(k, smem);
                if (r != cudaSuccess) return r;
                k<<<grid, fwd_threads<NW>(), smem, st>>>(mQ, mK, mV, mO32, mO, s, Qidx, Kidx, bd, tau, ptr, idx,
                                                         (TO*)O, O32, rownorm, split, err);
                note_launch();
                return cudaGetLastError();
            };
            constexpr int PI = decltype(ac)::pinv;
            if (fwd_wide(s)) return go(k3_forward<D, TO, PI, 4>, std::integral_constant<int, 4>{});
            return go(k3_forward<D, TO, PI, 2>, std::integral_constant<int, 2>{});
        });
    });
}

#endif  // part 2

#if ASA_PART(5)
// k <= 8: there the fused kernel (four epilogue warpgroups in both phases)
// is as fast as the separate launches; for k <= 16 the separate forward with
// two warpgroups is faster than either four-warpgroup variant.
bool tc_fused_supported(const Shape& s) {
    return !s.exact_tau && s.out_dtype == ASA_DTYPE_BF16 && s.k <= 8;
}

cudaError_t tc_fused_forward(const Shape& s, const void* Q, const void* K, const void* V, const int32_t* Qidx,
                             const int32_t* Kidx, float* tau, uint8_t* M, void* O, float* O32, float* rownorm,
                             void* ws, int* err, cudaStream_t st) {
    if (!tc_fused_supported(s)) return cudaErrorInvalidValue;
    cudaError_t e = launch_bounds(s, Qidx, Kidx, ws, st);
    if (e != cudaSuccess) return e;
    CUtensorMap mQ, mK, mV, mO32, mO;
    if (!make_map(&mQ, Q, s.BH, s.NQ, s.d) || !make_map(&mK, K, s.BH, s.NK, s.d) ||
        !make_map(&mV, V, s.BH, s.NK, s.d) ||
        !make_store_map(&mO, O, s.BH, s.NQ, s.d, s.out_dtype == ASA_DTYPE_F32))
        return cudaErrorInvalidValue;
    if (!O32) mO32 = mO;   // not stored
    else if (!make_store_map(&mO32, O32, s.BH, s.NQ, s.d, true)) return cudaErrorInvalidValue;
    Bounds bd = bounds_at(s, ws);
    dim3 grid(s.BH * s.nQB);
    const int split = s.split;
    using bf = __nv_bfloat16;
    return with_alpha(s, [&](auto ac) -> cudaError_t {
        constexpr int PI = decltype(ac)::pinv;
        auto go = [&](auto k, auto dtag, auto nw) -> cudaError_t {
            constexpr int D = decltype(dtag)::value, NW = decltype(nw)::value;
            // Q, K stages, the phase region, 48 barriers + TMEM holder, row
            // sums, τ, positions, counts, two schedules and the flags
            const size_t smem = (size_t)D * TILE * 2 * (1 + MASK_S) + fused_region_bytes<D, NW>() + 48 * 8 + 16 +
                                (size_t)(NW + 2) * TILE * 4 + 16 * 4 + (size_t)s.nKB * 9 + 64;
            cudaError_t r = prep(k, smem);
            if (r != cudaSuccess) return r;
            k<<<grid, fwd_threads<NW>(), smem, st>>>(mQ, mK, mV, mO32, mO, s, Qidx, Kidx, bd, tau, M, (bf*)O, O32,
                                                     rownorm, split, err);
            note_launch();
            return cudaGetLastError();
        };
        using I64 = std::integral_constant<int, 64>;
        using I128 = std::integral_constant<int, 128>;
        using W4 = std::integral_constant<int, 4>;
        if (s.d == 128) return go(k13_fused<128, bf, 8, PI, 4>, I128{}, W4{});
        return go(k13_fused<64, bf, 8, PI, 4>, I64{}, W4{});
    });
}
#endif  // part 5

// Backward launch arguments shared by the dQ and dK/dV launchers.
struct BwdArgs {
    CUtensorMap mQ, mK, mV, mdO;
    Bounds bd;
    const int32_t *Qidx, *Kidx, *ptr, *idx, *cptr, *cidx;
    const float *tau, *invNv, *Dq;
    void *dQ, *dK, *dV;
    int* err;
};

template <typename TO>
size_t bwd_smem(const Shape& s, int D) {
    return (size_t)D * TILE * 2 * 6 + kSmemTailBwd + (size_t)(s.nKB > s.nQB ? s.nKB : s.nQB) * 4;
}

cudaError_t tc_launch_dq(const Shape& s, const BwdArgs& a, cudaStream_t st);
cudaError_t tc_launch_dkdv(const Shape& s, const BwdArgs& a, cudaStream_t st);

#if ASA_PART(3)
cudaError_t tc_launch_dq(const Shape& s, const BwdArgs& a, cudaStream_t st) {
    const int split = s.split;
    return with_dtype_d(s, [&](auto dtag, auto* out) -> cudaError_t {
        constexpr int D = decltype(dtag)::value;
        using TO = std::remove_pointer_t<decltype(out)>;
        return with_alpha(s, [&](auto ac) -> cudaError_t {
            // Q, dO, three K stages, SV V stages, barriers/holder (256 B),
            // block positions (512 B), the tile schedule
            auto smem_for = [&](int sv) { return (size_t)D * TILE * 2 * (5 + sv) + 256 + 512 + (size_t)s.nKB * 4; };
            const bool two = smem_for(2) <= 232448;
            auto kdq = two ? k4_dq<D, TO, decltype(ac)::pe2, 2> : k4_dq<D, TO, decltype(ac)::pe2, 1>;
            const size_t smem = smem_for(two ? 2 : 1);
            cudaError_t r = prep(kdq, smem);
            if (r != cudaSuccess) return r;
            kdq<<<dim3(s.BH * s.nQB), DQ_THREADS, smem, st>>>(a.mQ, a.mK, a.mV, a.mdO, s, a.Qidx, a.Kidx, a.bd,
                                                             a.tau, a.invNv, a.Dq, a.ptr, a.idx, (TO*)a.dQ,
                                                             split, a.err);
            note_launch();
            return cudaGetLastError();
        });
    });
}

cudaError_t tc_backward(const Shape& s, const void* Q, const void* K, const void* V, const int32_t* Qidx,
                        const int32_t* Kidx, const float* O32, const float* tau, const int32_t* ptr,
                        const int32_t* idx, const int32_t* cptr, const int32_t* cidx,
                        const float* rownorm, const void* dO, void* dQ, void* dK, void* dV, void* ws,
                        int* err, cudaStream_t st, int stages) {
    BwdArgs a;
    a.bd = bounds_at(s, ws);
    float* Dq = (float*)((char*)ws + ((bounds_ints(s) * 4 + 15) & ~size_t(15)));
    const size_t rows = (size_t)s.BH * s.NQ;
    float* invNv = Dq + rows;
    cudaError_t e = cudaSuccess;
    const bool maps = make_map(&a.mQ, Q, s.BH, s.NQ, s.d) && make_map(&a.mK, K, s.BH, s.NK, s.d) &&
                      make_map(&a.mV, V, s.BH, s.NK, s.d) && make_map(&a.mdO, dO, s.BH, s.NQ, s.d);
    if (!maps && (stages & 6 || s.jacobian)) return cudaErrorInvalidValue;
    if (stages & 1) {
        // k4_pre reads O (fp32) and dO (bf16) rows as 16- and 8-byte vectors
        if (((uintptr_t)O32 & 15) || ((uintptr_t)dO & 15)) return cudaErrorInvalidValue;
        e = launch_bounds(s, Qidx, Kidx, ws, st);
        if (e != cudaSuccess) return e;
        if (s.d == 128)
            k4_pre<128><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(O32, (const __nv_bfloat16*)dO, rownorm, Dq,
                                                                     invNv, rows);
        else
            k4_pre<64><<<(unsigned)((rows + 15) / 16), 256, 0, st>>>(O32, (const __nv_bfloat16*)dO, rownorm, Dq,
                                                                    invNv, rows);
        note_launch();
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        if (s.jacobian) {
            // the Jacobian's row statistic replaces D = O·dO
            const Bounds bd = bounds_at(s, ws);
            e = with_alpha(s, [&](auto ac) -> cudaError_t {
                auto go = [&](auto kern, int D) -> cudaError_t {
                    const size_t smem = (size_t)D * TILE * 2 * 6 + (size_t)2 * DQ_NW * TILE * 4 + 24 * 8 + 16 +
                                        TILE * 4 + (size_t)s.nKB * 4 + 64;
                    cudaError_t r = prep(kern, smem);
                    if (r != cudaSuccess) return r;
                    kern<<<dim3(s.BH * s.nQB), DQ_THREADS, smem, st>>>(a.mQ, a.mK, a.mV, a.mdO, s, Qidx, Kidx, bd,
                                                                     tau, ptr, idx, Dq, err);
                    note_launch();
                    return cudaGetLastError();
                };
                if (s.d == 128) return go(k4_jac<128, decltype(ac)::pe2>, 128);
                return go(k4_jac<64, decltype(ac)::pe2>, 64);
            });
            if (e != cudaSuccess) return e;
        }
    }
    if (!(stages & 6)) return cudaSuccess;
    a.Qidx = Qidx; a.Kidx = Kidx; a.ptr = ptr; a.idx = idx; a.cptr = cptr; a.cidx = cidx;
    a.tau = tau; a.invNv = invNv; a.Dq = Dq; a.dQ = dQ; a.dK = dK; a.dV = dV; a.err = err;
    if (stages & 2) {
        e = tc_launch_dq(s, a, st);
        if (e != cudaSuccess) return e;
    }
    if (stages & 4) e = tc_launch_dkdv(s, a, st);
    return e;
}
#endif  // part 3

#if ASA_PART(4)
cudaError_t tc_launch_dkdv(const Shape& s, const BwdArgs& a, cudaStream_t st) {
    const int split = s.split;
    return with_dtype_d(s, [&](auto dtag, auto* out) -> cudaError_t {
        constexpr int D = decltype(dtag)::value;
        using TO = std::remove_pointer_t<decltype(out)>;
        return with_alpha(s, [&](auto ac) -> cudaError_t {
            auto kkv = k4_dkdv<D, TO, decltype(ac)::pinv, decltype(ac)::pe2>;
            const size_t smem = bwd_smem<TO>(s, D);
            cudaError_t r = prep(kkv, smem);
            if (r != cudaSuccess) return r;
            kkv<<<dim3(s.BH * s.nKB), DKV_THREADS, smem, st>>>(a.mQ, a.mK, a.mV, a.mdO, s, a.Qidx, a.Kidx, a.bd,
                                                          a.tau, a.invNv, a.Dq, a.cptr, a.cidx, (TO*)a.dK,
                                                          (TO*)a.dV, split, a.err);
            note_launch();
            return cudaGetLastError();
        });
    });
}
#endif  // part 4

}  // namespace asa

