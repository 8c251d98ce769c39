/*
 * asa.h -- C ABI of the B200 α-entmax block-sparse attention engine
 * (AdaSplash path: τ solve -> block mask / tile lists -> block-sparse forward
 * -> backward).
 *
 * Every entry point takes raw device pointers, sizes in an asa_params block
 * and a CUDA stream; it allocates nothing, never synchronises the device and
 * returns an asa_status code.  The caller owns every buffer, including the
 * workspace whose size asa_workspace_bytes() reports.  Calls are
 * stream-ordered and reentrant; they run on the device that is current on
 * the calling thread.
 *
 * Layouts (all contiguous, row-major):
 *   Q, dO, O, dQ        [B*H, NQ, d]   in_dtype / out_dtype
 *   K, V, dK, dV        [B*H, NK, d]
 *   Q_idx / K_idx       int32 [B*H, NQ] / [B*H, NK]  (key visible iff
 *                       K_idx <= Q_idx when causal)
 *   tau, rownorm        float [B*H, NQ]
 *   M                   uint8 [B*H, nQB, nKB], nQB = ceil(NQ/block_m),
 *                       nKB = ceil(NK/block_n)
 *   csr_ptr / csr_idx   int32 [B*H, nQB+1] / [B*H, nQB*nKB] (zero padded)
 *
 * Reference interfaces replaced (mvideet/Adaptive-Splash-Attention,
 * source/adasplashattention.cu):
 *   asa_tau_mask  <- build_mask_kernel + build_lookup_kernel launches inside
 *                    forward_splash (:580-591)
 *   asa_forward   <- forward_splash (:537-609), pybind "forward" (:703)
 *   asa_backward  <- backward_splash (:611-700), pybind "backward" (:704)
 *   asa_scrub     <- the host NaN/Inf scrub (:599-606, :684-697)
 */
#ifndef ASA_H_
#define ASA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* asa_stream_t; /* identical to cudaStream_t */

enum asa_status {
    ASA_OK = 0,
    ASA_ERR_INVALID = 1,        /* bad argument, shape or null pointer            */
    ASA_ERR_UNSUPPORTED = 2,    /* valid but not implemented (d > 128, ...)       */
    ASA_ERR_WORKSPACE = 3,      /* workspace too small                            */
    ASA_ERR_CUDA = 4,           /* a CUDA runtime call or launch failed           */
    ASA_ERR_DEVICE_TIMEOUT = 5  /* a kernel's bounded wait ran out (device error) */
};

enum asa_dtype { ASA_DTYPE_F32 = 0, ASA_DTYPE_BF16 = 1 };

enum asa_backend {
    ASA_BACKEND_AUTO = 0,  /* tcgen05 where the shape allows it, else SIMT   */
    ASA_BACKEND_SIMT = 1,  /* CUDA-core kernels in the reference's summation order */
    ASA_BACKEND_TC = 2     /* tcgen05 / TMEM / TMA kernels (bf16, d in {64,128}, 128x128 tiles) */
};

enum asa_tau_mode {
    ASA_TAU_REFERENCE = 0, /* the reference's τ: five Halley steps over the row's top-k, and   */
                           /* the mask = union of the block's top-k key blocks (:150-217)       */
    ASA_TAU_EXACT = 1      /* the exact α-entmax threshold over all of the row's visible keys */
                           /* (Σ [(α-1)s - τ]_+^{1/(α-1)} = 1), and the mask = every tile in   */
                           /* which some row of the block has a positive weight ("tile max vs */
                           /* τ"); the reference's tile-load zeroing does not apply           */
};

enum asa_grad_mode {
    ASA_GRAD_REFERENCE = 0, /* the reference's fixed-τ gradient (:481-507)                     */
    ASA_GRAD_JACOBIAN = 1   /* the α-entmax Jacobian: τ moves with the scores so that the row  */
                            /* mass Σp is held fixed -- g_i = w_i (dP_i - Σ_j w_j dP_j / Σ_j w_j) */
                            /* / Σp, w = ((α-1)s - τ)_+^{(2-α)/(α-1)}; with ASA_TAU_EXACT this */
                            /* is the exact gradient of α-entmax attention                    */
};

enum asa_precision {
    ASA_PREC_SPLIT = 0,    /* P and dS enter the tensor cores as bf16 hi+lo pairs (parity) */
    ASA_PREC_BF16 = 1      /* single bf16 P and dS (FlashAttention-style rounding)          */
};

typedef struct asa_params {
    int B, H;              /* batch and heads: B*H independent rows              */
    int NQ, NK, d;         /* query length, key length, head dim (<= 128)        */
    int block_m, block_n;  /* mask tile (reference BLOCK_M / BLOCK_N, :8-13)     */
    int k_keep;            /* top-k kept per query (reference K_KEEP, :17-19)    */
    float alpha;           /* entmax α, clamped to [1.05, 3] as the reference does (:547) */
    float sm_scale;        /* score scale                                        */
    int causal;            /* 1: key visible iff K_idx <= Q_idx; 0: all visible  */
    int in_dtype;          /* asa_dtype of Q, K, V, dO                           */
    int out_dtype;         /* asa_dtype of O, dQ, dK, dV                         */
    int backend;           /* asa_backend                                        */
    int precision;         /* asa_precision (tcgen05 backend only)               */
    long long timeout_spins; /* bound on every device-side wait; 0 = default     */
    int ref_tile_load;     /* 1 (default): reproduce the reference's tile-load   */
                           /* zeroing -- each K/V tile element is zeroed when the */
                           /* reference thread that stages it (query             */
                           /* qb*block_m + (col*d + dim) % block_m) cannot see    */
                           /* that key (:176-183, :285-294, :398-406, :442-450);  */
                           /* 0: every visible key is read in full.              */
    int tau_mode;          /* asa_tau_mode (default ASA_TAU_REFERENCE)            */
    int grad_mode;         /* asa_grad_mode (default ASA_GRAD_REFERENCE)          */
    int fused_forward;     /* tcgen05 forward with reference τ, bf16 out, k <= 8:  */
                           /* 1 (default) one kernel per query block runs τ /     */
                           /* mask and the forward (Q read once, no tile lists    */
                           /* between them); 0: separate τ / mask, tile-list and  */
                           /* forward launches.  Same outputs either way.         */
} asa_params;

/* Defaults: block 128x128, k_keep 8, α 1.5, sm_scale 0 (set it), causal,
 * bf16 in / bf16 out, AUTO backend, SPLIT precision, ref_tile_load 1,
 * reference τ and gradient, fused_forward 1. */
void asa_params_default(asa_params* p);

/* Workspace each call needs, in bytes (16-byte multiples).
 * Reference: forward_splash / backward_splash allocate these temporaries per
 * call with torch::zeros (:561-567, :640-649); here the caller does. */
int asa_workspace_bytes(const asa_params* p, size_t* fwd_bytes, size_t* bwd_bytes);

/* Which backend AUTO resolves to for p (ASA_BACKEND_SIMT or ASA_BACKEND_TC),
 * or a negative asa_status if p is invalid. */
int asa_resolve_backend(const asa_params* p);

/* τ per query and the block mask M, plus its CSR (reference build_mask_kernel
 * :150-217 and build_lookup_kernel :219-242).  csr_ptr / csr_idx may be NULL. */
int asa_tau_mask(const asa_params* p, const void* Q, const void* K,
                 const int32_t* Q_idx, const int32_t* K_idx,
                 float* tau, uint8_t* M, int32_t* csr_ptr, int32_t* csr_idx,
                 void* ws, size_t ws_bytes, asa_stream_t stream);

/* asa_tau_mask without a workspace argument: the same τ, block mask and CSR,
 * for callers that cannot allocate device memory (a plugin inside a host
 * framework whose allocator forbids cudaMalloc, or an embedded runtime that
 * owns all device memory up front).  No counterpart in the reference, which
 * allocates its temporaries with torch::zeros on every call.
 *
 * Scratch comes from a fixed device array of ASA_NOALLOC_SCRATCH_BYTES inside
 * the library (present on every GPU that loads it until the process exits);
 * shapes whose scratch need (asa_workspace_bytes' fwd_bytes) exceeds it are
 * rejected with ASA_ERR_WORKSPACE before anything is launched.  The first
 * call on each device looks the array's address up (cudaGetSymbolAddress);
 * make that first call before any stream capture.  Calls share the one
 * array, so two calls that overlap on the GPU (different streams, or
 * different host threads) race; serialise them.  Nothing is allocated: no
 * cudaMalloc, cudaFree or allocating library call. */
#define ASA_NOALLOC_SCRATCH_BYTES (1u << 20)
int asa_tau_mask_noalloc(const asa_params* p, const void* Q, const void* K,
                         const int32_t* Q_idx, const int32_t* K_idx,
                         float* tau, uint8_t* M, int32_t* csr_ptr, int32_t* csr_idx,
                         asa_stream_t stream);

/* Full forward: τ / mask / CSR, then O = Σ p v / (Σ p + 1e-8) over the active
 * tiles (reference forward_splash :537-609 and splash_forward_sparse
 * :244-341).  O is out_dtype; O32 (optional, may be NULL or equal to O when
 * out_dtype is F32) receives an fp32 copy for the backward; rownorm receives
 * Σ p per query.  tau, M, csr_ptr, csr_idx, rownorm are outputs the backward
 * consumes. */
int asa_forward(const asa_params* p, const void* Q, const void* K, const void* V,
                const int32_t* Q_idx, const int32_t* K_idx,
                void* O, float* O32, float* tau, uint8_t* M,
                int32_t* csr_ptr, int32_t* csr_idx, float* rownorm,
                void* ws, size_t ws_bytes, asa_stream_t stream);

/* Backward of the fixed-τ objective (reference splash_backward_sparse
 * :343-535) from the forward's saved tau / M / CSR / rownorm and its fp32
 * output O32.  dQ, dK, dV are out_dtype and fully overwritten
 * (deterministic: no atomics). */
int asa_backward(const asa_params* p, const void* Q, const void* K, const void* V,
                 const int32_t* Q_idx, const int32_t* K_idx,
                 const float* O32, const float* tau, const uint8_t* M,
                 const int32_t* csr_ptr, const int32_t* csr_idx, const float* rownorm,
                 const void* dO, void* dQ, void* dK, void* dV,
                 void* ws, size_t ws_bytes, asa_stream_t stream);

/* The top-k-only ("stable") operator of the reference notebook
 * (AdaSplashNotebook.ipynb file lines 303-450: stable_entmax_threshold,
 * stable_splash_kernel, stable_forward): per query the top-k clamped scores
 * of the visible keys (k_keep; the same top-k as asa_tau_mask, with no
 * tile-load zeroing), τ by five bisection steps (α clamped to [1.01, 3]),
 * the weights p_j / max(Σp, EPS) and O = Σ_j w_j V[key_j].  block_m/block_n
 * only choose the kernels of the top-k pass (128x128 with bf16 and d in
 * {64, 128}: tcgen05).  Outputs besides O, kept for the backward, are
 * [B*H*NQ*k] top_val (clamped scores, descending) and top_idx (keys, -1 for
 * a row with fewer visible keys), weights, and per row tau and tau_coef (the
 * weight of the bisection's upper start in τ). */
int asa_stable_workspace_bytes(const asa_params* p, size_t* fwd_bytes, size_t* bwd_bytes);
int asa_stable_forward(const asa_params* p, const void* Q, const void* K, const void* V,
                       const int32_t* Q_idx, const int32_t* K_idx, void* O, float* top_val,
                       int32_t* top_idx, float* weights, float* tau, float* tau_coef,
                       void* ws, size_t ws_bytes, asa_stream_t stream);

/* Gradient of asa_stable_forward (the notebook's stable_backward returns
 * zeros, nb:470-476): τ enters through the bisection's starting bracket,
 * whose ends depend on the largest and smallest kept score; a clamped score
 * passes no gradient.  dQ, dK, dV are out_dtype and fully overwritten; dK
 * and dV are gathered with fp32 atomics, so their last bits can vary run to
 * run. */
int asa_stable_backward(const asa_params* p, const void* Q, const void* K, const void* V,
                        const float* top_val, const int32_t* top_idx, const float* weights,
                        const float* tau, const float* tau_coef, const void* dO, void* dQ,
                        void* dK, void* dV, void* ws, size_t ws_bytes, asa_stream_t stream);

/* The reference's host-side scrub done on the device: NaN -> 0, and if any
 * element is ±Inf the whole tensor is clamped to [-100, 100]
 * (:599-606, :684-697).  ws needs 16 bytes. */
int asa_scrub(int dtype, void* x, size_t n, void* ws, asa_stream_t stream);

/* Reads (and clears) the device error word the kernels set when a bounded
 * wait runs out.  Synchronises the stream.  *code is 0 when no error. */
int asa_device_error(asa_stream_t stream, int* code);

/* Enqueues on `stream` a copy of the device error word into *host_word
 * (pinned host memory, for the copy to stay asynchronous) without clearing
 * it or synchronising: a caller checks the value after a later
 * synchronisation point and then reads and clears the word with
 * asa_device_error.  No counterpart in the reference, whose host launchers
 * synchronise and raise after every call (CUDA_CHECK, :24-27). */
int asa_device_error_async(asa_stream_t stream, int* host_word);

/* Self-test of the device-side timeout path: launches one block whose wait
 * on a barrier phase that nothing completes gives up after `spins` polls and
 * records ASA_ERR_DEVICE_TIMEOUT in the device error word (read it with
 * asa_device_error).  The kernel returns on its own and leaves no work in
 * flight.  No counterpart in the reference. */
int asa_wait_probe(long long spins, asa_stream_t stream);

/* Per-launch timing for benchmarks and tracing (no counterpart in the
 * reference, which only wall-clocks whole calls, nb:1791-1796).
 * asa_profile_begin(1) makes every entry point record a CUDA event before
 * and after each kernel it launches on its stream; asa_profile_end()
 * synchronises on those events and aggregates per kernel label; then
 * asa_profile_get(i, ...) returns label i's total milliseconds and launch
 * count (ASA_ERR_INVALID past the last label).  Recording is process-wide
 * (launches from every host thread).  asa_launch_count() is the number of kernels the library has
 * launched since load. */
int asa_profile_begin(int enable);
int asa_profile_end(void);
int asa_profile_get(int i, const char** label, double* total_ms, int* launches);
long long asa_launch_count(void);

/* Text of the CUDA error behind the calling thread's last ASA_ERR_CUDA. */
const char* asa_last_cuda_error(void);

/* Human-readable text of an asa_status. */
const char* asa_status_string(int status);

/* ABI version: major*10000 + minor*100 + patch. */
int asa_version(void);

#ifdef __cplusplus
}
#endif
#endif /* ASA_H_ */
