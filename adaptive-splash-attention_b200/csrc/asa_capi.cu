// asa_capi.cu -- the extern "C" entry points declared in include/asa.h:
// argument checks, workspace layout, backend choice and launch order.
//
// Reference host launchers replaced: forward_splash / backward_splash
// (source/adasplashattention.cu:537-700).  Differences by design: nothing is
// allocated here (the caller passes every buffer), nothing synchronises the
// device, launches go on the caller's stream, and errors come back as status
// codes instead of exceptions.
#include "asa_internal.h"
#include "asa_sm100.cuh"
#include <atomic>
#include <mutex>
#include <climits>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

namespace asa {
// tcgen05 kernels (asa_tc.cu)
bool tc_supported(const Shape& s);
size_t tc_fwd_workspace(const Shape& s);
size_t tc_bwd_workspace(const Shape& s);
cudaError_t tc_tau_mask(const Shape& s, const void* Q, const void* K, const int32_t* Qidx,
                        const int32_t* Kidx, float* tau, uint8_t* M, void* ws, int* err,
                        cudaStream_t st, float* topv_out = nullptr, int32_t* topi_out = nullptr);
cudaError_t tc_exact_tau(const Shape& s, const void* Q, const void* K, const int32_t* Qidx,
                         const int32_t* Kidx, float* tau, uint8_t* M, void* ws, int* err,
                         cudaStream_t st);
cudaError_t tc_forward(const Shape& s, const void* Q, const void* K, const void* V,
                       const int32_t* Qidx, const int32_t* Kidx, const float* tau,
                       const int32_t* ptr, const int32_t* idx, void* O, float* O32,
                       float* rownorm, void* ws, int* err, cudaStream_t st);
bool tc_fused_supported(const Shape& s);
cudaError_t tc_fused_forward(const Shape& s, const void* Q, const void* K, const void* V,
                             const int32_t* Qidx, const int32_t* Kidx, float* tau, uint8_t* M,
                             void* O, float* O32, float* rownorm, void* ws, int* err, cudaStream_t st);
cudaError_t tc_backward(const Shape& s, const void* Q, const void* K, const void* V,
                        const int32_t* Qidx, const int32_t* Kidx, const float* O32,
                        const float* tau, const int32_t* ptr, const int32_t* idx,
                        const int32_t* cptr, const int32_t* cidx, const float* rownorm,
                        const void* dO, void* dQ, void* dK, void* dV, void* ws, int* err,
                        cudaStream_t st, int stages);
}  // namespace asa

__device__ int g_asa_error;

namespace {
std::atomic<long long> g_launches{0};
}
void asa::note_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

namespace {

// ---- launch profiler: events around each internal launch (per host thread)
struct ProfMark {
    const char* label;
    cudaEvent_t start, stop;
    long long launches;
};
struct ProfState {
    bool on = false;
    std::vector<ProfMark> marks;
    std::vector<std::string> labels;
    std::vector<double> ms;
    std::vector<int> counts;
};
ProfState g_prof;
std::mutex g_prof_mu;

// Scope that times everything launched on `st` between its construction and
// destruction under `label` when profiling is on.
struct ProfScope {
    ProfMark m{};
    cudaStream_t st;
    bool on;
    ProfScope(const char* label, cudaStream_t s) : st(s), on(g_prof.on) {
        if (!on) return;
        m.label = label;
        m.launches = g_launches.load();
        cudaEventCreate(&m.start);
        cudaEventCreate(&m.stop);
        cudaEventRecord(m.start, st);
    }
    ~ProfScope() {
        if (!on) return;
        cudaEventRecord(m.stop, st);
        m.launches = g_launches.load() - m.launches;
        std::lock_guard<std::mutex> lk(g_prof_mu);
        g_prof.marks.push_back(m);
    }
};


using asa::Shape;

constexpr int kMaxDevices = 64;
// Per-device addresses of device symbols, looked up once per device.  Host
// threads may race on the first lookup; each writes the same value, and the
// atomics make that race well defined.
std::atomic<int*> g_err_ptr[kMaxDevices];

int* error_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    int* w = g_err_ptr[dev].load(std::memory_order_relaxed);
    if (!w) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_asa_error) != cudaSuccess) return nullptr;
        w = (int*)p;
        g_err_ptr[dev].store(w, std::memory_order_relaxed);
    }
    return w;
}

size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

int check_params(const asa_params* p) {
    if (!p) return ASA_ERR_INVALID;
    if (p->B < 1 || p->H < 1 || p->NQ < 0 || p->NK < 0) return ASA_ERR_INVALID;
    if (p->d < 1 || p->block_m < 1 || p->block_n < 1) return ASA_ERR_INVALID;
    if (p->k_keep < 1 || p->k_keep > p->block_n) return ASA_ERR_INVALID;   // reference :32
    if (!std::isfinite(p->alpha) || !std::isfinite(p->sm_scale)) return ASA_ERR_INVALID;
    if ((p->in_dtype != ASA_DTYPE_F32 && p->in_dtype != ASA_DTYPE_BF16) ||
        (p->out_dtype != ASA_DTYPE_F32 && p->out_dtype != ASA_DTYPE_BF16))
        return ASA_ERR_INVALID;
    if (p->backend < ASA_BACKEND_AUTO || p->backend > ASA_BACKEND_TC) return ASA_ERR_INVALID;
    if (p->precision != ASA_PREC_SPLIT && p->precision != ASA_PREC_BF16) return ASA_ERR_INVALID;
    if (p->tau_mode != ASA_TAU_REFERENCE && p->tau_mode != ASA_TAU_EXACT) return ASA_ERR_INVALID;
    if (p->grad_mode != ASA_GRAD_REFERENCE && p->grad_mode != ASA_GRAD_JACOBIAN) return ASA_ERR_INVALID;
    if (p->fused_forward != 0 && p->fused_forward != 1) return ASA_ERR_INVALID;
    if (p->d > 128) return ASA_ERR_UNSUPPORTED;        // reference D_MAX (:14-16)
    if (p->k_keep > 32) return ASA_ERR_UNSUPPORTED;
    const long long BH = (long long)p->B * p->H;
    if (BH > INT_MAX / 2 || BH * p->NQ * p->d > (1LL << 40) || BH * p->NK * p->d > (1LL << 40))
        return ASA_ERR_UNSUPPORTED;
    return ASA_OK;
}

Shape make_shape(const asa_params* p) {
    Shape s;
    s.BH = p->B * p->H;
    s.NQ = p->NQ;
    s.NK = p->NK;
    s.d = p->d;
    s.BM = p->block_m;
    s.BN = p->block_n;
    s.k = p->k_keep;
    s.causal = p->causal ? 1 : 0;
    s.nQB = (p->NQ + p->block_m - 1) / p->block_m;
    s.nKB = (p->NK + p->block_n - 1) / p->block_n;
    s.alpha = std::fmax(1.05f, std::fmin(p->alpha, 3.0f));               // :547
    s.am1 = s.alpha - 1.0f;
    s.inv_am1b = 1.0f / (s.alpha - 1.0f);
    s.scale = p->sm_scale;
    s.pinv = asa::make_pow(1.0f / s.am1);
    s.pe2 = asa::make_pow((2.0f - s.alpha) / (s.alpha - 1.0f));          // :495
    s.spins = p->timeout_spins > 0 ? p->timeout_spins : (1LL << 22);
    s.in_dtype = p->in_dtype;
    s.out_dtype = p->out_dtype;
    s.exact_tau = p->tau_mode == ASA_TAU_EXACT ? 1 : 0;
    s.jacobian = p->grad_mode == ASA_GRAD_JACOBIAN ? 1 : 0;
    // the exact threshold is a property of the rows as given: no tile-load zeroing
    s.ref_load = (p->ref_tile_load && p->causal && !s.exact_tau) ? 1 : 0;
    s.split = p->precision == ASA_PREC_SPLIT ? 1 : 0;
    return s;
}

int resolve(const asa_params* p, const Shape& s) {
    if (p->backend == ASA_BACKEND_SIMT) return ASA_BACKEND_SIMT;
    const bool tc = asa::tc_supported(s);
    if (p->backend == ASA_BACKEND_TC) return tc ? ASA_BACKEND_TC : -ASA_ERR_UNSUPPORTED;
    return tc ? ASA_BACKEND_TC : ASA_BACKEND_SIMT;
}

// Backward workspace: [invN | accdO | csc_ptr | csc_idx | backend extra]
struct BwdLayout {
    size_t invN, accdO, cptr, cidx, extra, total;
};
BwdLayout bwd_layout(const Shape& s, int backend) {
    BwdLayout L;
    size_t o = 0;
    const size_t rows = (size_t)s.BH * s.NQ;
    L.invN = o; o = align16(o + rows * 4);
    L.accdO = o; o = align16(o + rows * 4);
    L.cptr = o; o = align16(o + (size_t)s.BH * (s.nKB + 1) * 4);
    L.cidx = o; o = align16(o + (size_t)s.BH * s.nKB * s.nQB * 4);
    L.extra = o;
    if (backend == ASA_BACKEND_TC) o = align16(o + asa::tc_bwd_workspace(s));
    L.total = o + 16;
    return L;
}
size_t fwd_bytes(const Shape& s, int backend) {
    size_t o = 16;
    if (backend == ASA_BACKEND_TC) o = align16(o + asa::tc_fwd_workspace(s));
    return o;
}

thread_local cudaError_t g_last_cuda = cudaSuccess;

// asa_wait_probe's kernel: lane 0 waits, with the kernels' bounded wait, on
// phase 0 of a shared-memory mbarrier that expects one arrival nobody makes,
// so the wait runs out after `spins` polls and records
// ASA_ERR_DEVICE_TIMEOUT in the error word; then the barrier is completed by
// the thread itself, so nothing is left pending when the block exits.
__global__ void wait_probe_kernel(long long spins, int* err) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        asa::sm100::mbar_init(&bar, 1);
        asa::sm100::fence_barrier_init();
        asa::sm100::mbar_wait(&bar, 0, spins, err, ASA_ERR_DEVICE_TIMEOUT);
        asa::sm100::mbar_arrive(&bar);
    }
    __syncwarp();
}
int cuda_status(cudaError_t e) {
    if (e == cudaSuccess) return ASA_OK;
    g_last_cuda = e;
    return ASA_ERR_CUDA;
}

}  // namespace

extern "C" {

void asa_params_default(asa_params* p) {
    if (!p) return;
    std::memset(p, 0, sizeof(*p));
    p->B = p->H = 1;
    p->block_m = p->block_n = 128;
    p->k_keep = 8;
    p->alpha = 1.5f;
    p->causal = 1;
    p->in_dtype = ASA_DTYPE_BF16;
    p->out_dtype = ASA_DTYPE_BF16;
    p->backend = ASA_BACKEND_AUTO;
    p->precision = ASA_PREC_SPLIT;
    p->ref_tile_load = 1;
    p->tau_mode = ASA_TAU_REFERENCE;
    p->grad_mode = ASA_GRAD_REFERENCE;
    p->fused_forward = 1;
}

int asa_resolve_backend(const asa_params* p) {
    int rc = check_params(p);
    if (rc) return -rc;
    return resolve(p, make_shape(p));
}

int asa_workspace_bytes(const asa_params* p, size_t* fwd, size_t* bwd) {
    int rc = check_params(p);
    if (rc) return rc;
    Shape s = make_shape(p);
    int b = resolve(p, s);
    if (b < 0) return -b;
    if (fwd) *fwd = fwd_bytes(s, b);
    if (bwd) *bwd = bwd_layout(s, b).total;
    return ASA_OK;
}

int asa_tau_mask(const asa_params* p, const void* Q, const void* K, const int32_t* Qidx,
                 const int32_t* Kidx, float* tau, uint8_t* M, int32_t* csr_ptr, int32_t* csr_idx,
                 void* ws, size_t ws_bytes, asa_stream_t stream) {
    int rc = check_params(p);
    if (rc) return rc;
    Shape s = make_shape(p);
    int b = resolve(p, s);
    if (b < 0) return -b;
    if (s.NQ == 0) return ASA_OK;
    if (!Q || (!K && s.NK) || !tau || !M || (p->causal && (!Qidx || (!Kidx && s.NK))))
        return ASA_ERR_INVALID;
    if (ws_bytes < fwd_bytes(s, b) || !ws) return ASA_ERR_WORKSPACE;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e;
    {
        ProfScope ps("tau_mask", st);
        if (s.exact_tau)
            e = b == ASA_BACKEND_TC ? asa::tc_exact_tau(s, Q, K, Qidx, Kidx, tau, M, ws, error_word(), st)
                                    : asa::simt_exact_tau(s, Q, K, Qidx, Kidx, tau, M, st);
        else if (b == ASA_BACKEND_TC)
            e = asa::tc_tau_mask(s, Q, K, Qidx, Kidx, tau, M, ws, error_word(), st);
        else
            e = asa::simt_tau_mask(s, Q, K, Qidx, Kidx, tau, M, st);
    }
    if (e != cudaSuccess) return cuda_status(e);
    if (csr_ptr && csr_idx) {
        ProfScope ps("tile_lists", st);
        e = asa::build_lists(s, M, csr_ptr, csr_idx, nullptr, nullptr, st);
    }
    return cuda_status(e);
}

int asa_forward(const asa_params* p, const void* Q, const void* K, const void* V,
                const int32_t* Qidx, const int32_t* Kidx, void* O, float* O32, float* tau,
                uint8_t* M, int32_t* csr_ptr, int32_t* csr_idx, float* rownorm, void* ws,
                size_t ws_bytes, asa_stream_t stream) {
    int rc = check_params(p);
    if (rc) return rc;
    Shape s = make_shape(p);
    int b = resolve(p, s);
    if (b < 0) return -b;
    if (s.NQ == 0) return ASA_OK;
    if (!O || !csr_ptr || !csr_idx || !rownorm) return ASA_ERR_INVALID;
    if (!V && s.NK) return ASA_ERR_INVALID;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e;
    if (b == ASA_BACKEND_TC && p->fused_forward && asa::tc_fused_supported(s)) {
        // one kernel: τ / mask and the forward; the tile lists (an output the
        // backward reads) follow from the mask
        if (!Q || !K || !tau || !M || (p->causal && (!Qidx || !Kidx))) return ASA_ERR_INVALID;
        if (ws_bytes < fwd_bytes(s, b) || !ws) return ASA_ERR_WORKSPACE;
        {
            ProfScope ps("forward_fused", st);
            e = asa::tc_fused_forward(s, Q, K, V, Qidx, Kidx, tau, M, O, O32, rownorm, ws, error_word(), st);
        }
        if (e == cudaSuccess) {
            ProfScope ps("tile_lists", st);
            e = asa::build_lists(s, M, csr_ptr, csr_idx, nullptr, nullptr, st);
        }
        return cuda_status(e);
    }
    rc = asa_tau_mask(p, Q, K, Qidx, Kidx, tau, M, csr_ptr, csr_idx, ws, ws_bytes, stream);
    if (rc) return rc;
    ProfScope ps("forward", st);
    if (b == ASA_BACKEND_TC)
        e = asa::tc_forward(s, Q, K, V, Qidx, Kidx, tau, csr_ptr, csr_idx, O, O32, rownorm, ws,
                            error_word(), st);
    else
        e = asa::simt_forward(s, Q, K, V, Qidx, Kidx, tau, csr_ptr, csr_idx, O, O32, rownorm, st);
    return cuda_status(e);
}

int asa_backward(const asa_params* p, const void* Q, const void* K, const void* V,
                 const int32_t* Qidx, const int32_t* Kidx, const float* O32, const float* tau,
                 const uint8_t* M, const int32_t* csr_ptr, const int32_t* csr_idx,
                 const float* rownorm, const void* dO, void* dQ, void* dK, void* dV, void* ws,
                 size_t ws_bytes, asa_stream_t stream) {
    int rc = check_params(p);
    if (rc) return rc;
    Shape s = make_shape(p);
    int b = resolve(p, s);
    if (b < 0) return -b;
    if (!ws) return ASA_ERR_WORKSPACE;
    BwdLayout L = bwd_layout(s, b);
    if (ws_bytes < L.total) return ASA_ERR_WORKSPACE;
    cudaStream_t st = (cudaStream_t)stream;
    const size_t kbytes = (size_t)s.BH * s.NK * s.d * (p->out_dtype == ASA_DTYPE_F32 ? 4 : 2);
    if (s.NQ == 0) {   // no queries: every key gradient is zero
        if (kbytes) {
            if (!dK || !dV) return ASA_ERR_INVALID;
            cudaError_t e = cudaMemsetAsync(dK, 0, kbytes, st);
            if (e == cudaSuccess) e = cudaMemsetAsync(dV, 0, kbytes, st);
            return cuda_status(e);
        }
        return ASA_OK;
    }
    if (!Q || !dO || !dQ || !tau || !M || !csr_ptr || !csr_idx) return ASA_ERR_INVALID;
    if (s.NK && (!K || !V || !dK || !dV)) return ASA_ERR_INVALID;
    if (p->causal && (!Qidx || (!Kidx && s.NK))) return ASA_ERR_INVALID;
    char* w = (char*)ws;
    float* invN = (float*)(w + L.invN);
    float* accdO = (float*)(w + L.accdO);
    int32_t* cptr = (int32_t*)(w + L.cptr);
    int32_t* cidx = (int32_t*)(w + L.cidx);
    cudaError_t e;
    {
        ProfScope ps("tile_lists_t", st);
        e = asa::build_lists(s, M, nullptr, nullptr, cptr, cidx, st);
    }
    if (e != cudaSuccess) return cuda_status(e);
    if (b == ASA_BACKEND_TC) {
        if (!O32 || !rownorm) return ASA_ERR_INVALID;
        static const char* labels[3] = {"bwd_pre", "bwd_dq", "bwd_dkdv"};
        for (int k = 0; k < 3 && e == cudaSuccess; ++k) {
            ProfScope ps(labels[k], st);
            e = asa::tc_backward(s, Q, K, V, Qidx, Kidx, O32, tau, csr_ptr, csr_idx, cptr, cidx,
                                 rownorm, dO, dQ, dK, dV, w + L.extra, error_word(), st, 1 << k);
        }
        return cuda_status(e);
    }
    {
        ProfScope ps("bwd_rowstats", st);
        e = s.jacobian
                ? asa::simt_jacobian_stats(s, Q, K, V, Qidx, Kidx, tau, csr_ptr, csr_idx, dO, invN, accdO, st)
                : asa::simt_rowstats(s, Q, K, V, Qidx, Kidx, tau, csr_ptr, csr_idx, dO, invN, accdO, st);
    }
    if (e == cudaSuccess) {
        ProfScope ps("bwd_dq", st);
        e = asa::simt_dq(s, Q, K, V, Qidx, Kidx, tau, csr_ptr, csr_idx, dO, invN, accdO, dQ, st);
    }
    if (e == cudaSuccess && s.NK) {
        ProfScope ps("bwd_dkdv", st);
        e = asa::simt_dkdv(s, Q, K, V, Qidx, Kidx, tau, cptr, cidx, dO, invN, accdO, dK, dV, st);
    }
    return cuda_status(e);
}

// ---- allocation-free τ / block mask ------------------------------------------
// Some callers cannot allocate device memory at the point where they need
// the mask: code running inside another framework's custom allocator or
// memory pool that forbids cudaMalloc from a plugin, or an embedded host that
// has handed all device memory to a fixed arena.  For them
// asa_tau_mask_noalloc() takes its scratch from this file-scope device
// array instead of a caller workspace.  The array lives on every GPU that
// loads the library, for the life of the process.
static __device__ __align__(256) unsigned char g_asa_noalloc_scratch[ASA_NOALLOC_SCRATCH_BYTES];

namespace {
std::atomic<void*> g_noalloc_ptr[kMaxDevices];

// Device address of g_asa_noalloc_scratch on the current device.  Host code
// must not use the symbol itself (it names a host-side shadow); the address
// comes from cudaGetSymbolAddress, looked up once per device with that
// device current.
int noalloc_scratch(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_status(e);
    if (dev < 0 || dev >= kMaxDevices) return ASA_ERR_UNSUPPORTED;
    void* ptr = g_noalloc_ptr[dev].load(std::memory_order_relaxed);
    if (!ptr) {
        e = cudaGetSymbolAddress(&ptr, g_asa_noalloc_scratch);
        if (e != cudaSuccess) return cuda_status(e);
        g_noalloc_ptr[dev].store(ptr, std::memory_order_relaxed);
    }
    *out = ptr;
    return ASA_OK;
}
}  // namespace

int asa_tau_mask_noalloc(const asa_params* p, const void* Q, const void* K, const int32_t* Qidx,
                         const int32_t* Kidx, float* tau, uint8_t* M, int32_t* csr_ptr,
                         int32_t* csr_idx, asa_stream_t stream) {
    size_t need = 0;
    int rc = asa_workspace_bytes(p, &need, nullptr);
    if (rc) return rc;
    if (need > ASA_NOALLOC_SCRATCH_BYTES) return ASA_ERR_WORKSPACE;
    void* scratch = nullptr;
    rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    // Every call rewrites the part of the scratch it reads (the per-block
    // index bounds) before reading it, so nothing needs clearing here.
    return asa_tau_mask(p, Q, K, Qidx, Kidx, tau, M, csr_ptr, csr_idx, scratch,
                        ASA_NOALLOC_SCRATCH_BYTES, stream);
}

// ---- the top-k-only ("stable") operator ---------------------------------------
namespace {
// Forward workspace: [the τ/mask pass's workspace | M (unused by the operator)]
struct StableLayout {
    size_t mask, fwd, bwd;
};
StableLayout stable_layout(const Shape& s, int backend) {
    StableLayout L;
    L.mask = align16(fwd_bytes(s, backend));
    L.fwd = align16(L.mask + (size_t)s.BH * s.nQB * s.nKB);
    L.bwd = align16((size_t)2 * s.BH * s.NK * s.d * sizeof(float));   // fp32 dK, dV
    return L;
}
Shape stable_shape(const asa_params* p) {
    Shape s = make_shape(p);
    s.ref_load = 0;          // the notebook kernel reads K rows directly
    s.exact_tau = 0;
    return s;
}
}  // namespace

int asa_stable_workspace_bytes(const asa_params* p, size_t* fwd, size_t* bwd) {
    int rc = check_params(p);
    if (rc) return rc;
    Shape s = stable_shape(p);
    int b = resolve(p, s);
    if (b < 0) return -b;
    StableLayout L = stable_layout(s, b);
    if (fwd) *fwd = L.fwd;
    if (bwd) *bwd = L.bwd;
    return ASA_OK;
}

int asa_stable_forward(const asa_params* p, const void* Q, const void* K, const void* V,
                       const int32_t* Qidx, const int32_t* Kidx, void* O, float* top_val,
                       int32_t* top_idx, float* weights, float* tau, float* tau_coef, void* ws,
                       size_t ws_bytes, asa_stream_t stream) {
    int rc = check_params(p);
    if (rc) return rc;
    Shape s = stable_shape(p);
    int b = resolve(p, s);
    if (b < 0) return -b;
    if (s.NQ == 0) return ASA_OK;
    if (!Q || !O || !top_val || !top_idx || !weights || !tau || !tau_coef) return ASA_ERR_INVALID;
    if (s.NK && (!K || !V)) return ASA_ERR_INVALID;
    if (p->causal && (!Qidx || (!Kidx && s.NK))) return ASA_ERR_INVALID;
    StableLayout L = stable_layout(s, b);
    if (!ws || ws_bytes < L.fwd) return ASA_ERR_WORKSPACE;
    cudaStream_t st = (cudaStream_t)stream;
    uint8_t* M = (uint8_t*)ws + L.mask;
    cudaError_t e;
    {
        ProfScope ps("stable_topk", st);
        e = b == ASA_BACKEND_TC
                ? asa::tc_tau_mask(s, Q, K, Qidx, Kidx, nullptr, M, ws, error_word(), st, top_val, top_idx)
                : asa::simt_tau_mask(s, Q, K, Qidx, Kidx, nullptr, M, st, top_val, top_idx);
    }
    if (e != cudaSuccess) return cuda_status(e);
    ProfScope ps("stable_forward", st);
    return cuda_status(asa::stable_forward(s, p->alpha, V, top_val, top_idx, O, tau, weights, tau_coef, st));
}

int asa_stable_backward(const asa_params* p, const void* Q, const void* K, const void* V,
                        const float* top_val, const int32_t* top_idx, const float* weights,
                        const float* tau, const float* tau_coef, const void* dO, void* dQ, void* dK,
                        void* dV, void* ws, size_t ws_bytes, asa_stream_t stream) {
    int rc = check_params(p);
    if (rc) return rc;
    Shape s = stable_shape(p);
    int b = resolve(p, s);
    if (b < 0) return -b;
    StableLayout L = stable_layout(s, b);
    if (!ws || ws_bytes < L.bwd) return ASA_ERR_WORKSPACE;
    if (s.NQ && (!Q || !dO || !dQ || !top_val || !top_idx || !weights || !tau || !tau_coef))
        return ASA_ERR_INVALID;
    if (s.NK && (!K || !V || !dK || !dV)) return ASA_ERR_INVALID;
    float* dK32 = (float*)ws;
    float* dV32 = dK32 + (size_t)s.BH * s.NK * s.d;
    ProfScope ps("stable_backward", (cudaStream_t)stream);
    return cuda_status(asa::stable_backward(s, p->alpha, Q, K, V, dO, top_val, top_idx, weights, tau,
                                            tau_coef, dQ, dK32, dV32, dK, dV, (cudaStream_t)stream));
}

int asa_scrub(int dtype, void* x, size_t n, void* ws, asa_stream_t stream) {
    if ((dtype != ASA_DTYPE_F32 && dtype != ASA_DTYPE_BF16) || (n && !x) || !ws)
        return ASA_ERR_INVALID;
    return cuda_status(asa::scrub(dtype, x, n, (int*)ws, (cudaStream_t)stream));
}

int asa_device_error(asa_stream_t stream, int* code) {
    if (!code) return ASA_ERR_INVALID;
    int* w = error_word();
    if (!w) return ASA_ERR_CUDA;
    cudaStream_t st = (cudaStream_t)stream;
    int v = 0;
    cudaError_t e = cudaMemcpyAsync(&v, w, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e == cudaSuccess) e = cudaMemsetAsync(w, 0, sizeof(int), st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    *code = v;
    return cuda_status(e);
}

int asa_device_error_async(asa_stream_t stream, int* host_word) {
    if (!host_word) return ASA_ERR_INVALID;
    int* w = error_word();
    if (!w) return ASA_ERR_CUDA;
    return cuda_status(cudaMemcpyAsync(host_word, w, sizeof(int), cudaMemcpyDeviceToHost,
                                       (cudaStream_t)stream));
}

int asa_wait_probe(long long spins, asa_stream_t stream) {
    if (spins < 1) return ASA_ERR_INVALID;
    int* w = error_word();
    if (!w) return ASA_ERR_CUDA;
    wait_probe_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(spins, w);
    asa::note_launch();
    return cuda_status(cudaGetLastError());
}

int asa_profile_begin(int enable) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    for (auto& m : g_prof.marks) {
        cudaEventDestroy(m.start);
        cudaEventDestroy(m.stop);
    }
    g_prof.marks.clear();
    g_prof.labels.clear();
    g_prof.ms.clear();
    g_prof.counts.clear();
    g_prof.on = enable != 0;
    return ASA_OK;
}

int asa_profile_end(void) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    g_prof.on = false;
    int rc = ASA_OK;
    for (auto& m : g_prof.marks) {
        float ms = 0.0f;
        if (cudaEventSynchronize(m.stop) != cudaSuccess ||
            cudaEventElapsedTime(&ms, m.start, m.stop) != cudaSuccess)
            rc = ASA_ERR_CUDA;
        size_t i = 0;
        while (i < g_prof.labels.size() && g_prof.labels[i] != m.label) ++i;
        if (i == g_prof.labels.size()) {
            g_prof.labels.push_back(m.label);
            g_prof.ms.push_back(0.0);
            g_prof.counts.push_back(0);
        }
        g_prof.ms[i] += ms;
        g_prof.counts[i] += (int)m.launches;
        cudaEventDestroy(m.start);
        cudaEventDestroy(m.stop);
    }
    g_prof.marks.clear();
    return rc;
}

int asa_profile_get(int i, const char** label, double* total_ms, int* launches) {
    if (i < 0 || i >= (int)g_prof.labels.size()) return ASA_ERR_INVALID;
    if (label) *label = g_prof.labels[i].c_str();
    if (total_ms) *total_ms = g_prof.ms[i];
    if (launches) *launches = g_prof.counts[i];
    return ASA_OK;
}

long long asa_launch_count(void) { return g_launches.load(); }

const char* asa_last_cuda_error(void) { return cudaGetErrorString(g_last_cuda); }

const char* asa_status_string(int status) {
    switch (status) {
        case ASA_OK: return "ok";
        case ASA_ERR_INVALID: return "invalid argument";
        case ASA_ERR_UNSUPPORTED: return "unsupported configuration";
        case ASA_ERR_WORKSPACE: return "workspace too small";
        case ASA_ERR_CUDA: return "CUDA error";
        case ASA_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
        default: return "unknown status";
    }
}

int asa_version(void) { return 200; }

}  // extern "C"
