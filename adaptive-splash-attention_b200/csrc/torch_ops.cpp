// torch_ops.cpp -- the splash_attention operators registered with PyTorch's
// dispatcher (TORCH_LIBRARY), a thin layer over the C ABI of libasa.so.
//
// Reference binding replaced: the pybind module of
// source/adasplashattention.cu:702-705 (forward / backward).  Here the
// operators carry a schema, CUDA kernels that allocate their outputs and
// workspace with PyTorch's caching allocator and launch on the current
// stream, and Meta kernels (shapes only) so the operators can be traced.
// Autograd is attached on the Python side (torch.library.register_autograd).
//
//   splash_attention::forward(Q, K, V, Q_idx?, K_idx?, alpha, sm_scale, k_keep,
//       block_m, block_n, causal, backend, precision, out_f32, ref_tile_load,
//       tau_mode, grad_mode, fused_forward, need_o32)
//       -> (O, O32, tau, M, csr_ptr, csr_idx, rownorm)
//   splash_attention::backward(Q, K, V, Q_idx?, K_idx?, O32, tau, M, csr_ptr,
//       csr_idx, rownorm, dO, alpha, sm_scale, k_keep, block_m, block_n,
//       causal, backend, precision, out_f32, ref_tile_load, tau_mode,
//       grad_mode) -> (dQ, dK, dV)
//
// O32 is the fp32 copy of O the backward reads; it is empty when need_o32 is
// false (no backward will follow) and when O itself is fp32 (the backward
// then takes O as its O32).  Errors raise
// c10::Error (RuntimeError in Python), as the reference's TORCH_CHECKs do.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <mutex>
#include <string>

#include "../../include/asa.h"

namespace {

using at::Tensor;

void check(int rc, const char* what) {
    if (rc == ASA_OK) return;
    std::string msg = std::string(what) + ": " + asa_status_string(rc) + " (asa_status " +
                      std::to_string(rc) + ")";
    if (rc == ASA_ERR_CUDA) msg += std::string(": ") + asa_last_cuda_error();
    TORCH_CHECK(false, msg);
}

int dtype_code(at::ScalarType t) {
    if (t == at::kFloat) return ASA_DTYPE_F32;
    if (t == at::kBFloat16) return ASA_DTYPE_BF16;
    TORCH_CHECK(false, "splash_attention: unsupported dtype ", t, " (float32 or bfloat16)");
    return -1;
}

struct Cfg {
    double alpha, sm_scale;
    int64_t k_keep, block_m, block_n;
    bool causal;
    int64_t backend, precision;
    bool out_f32, ref_tile_load;
    int64_t tau_mode, grad_mode;
};

asa_params make_params(const Tensor& Q, const Tensor& K, const Cfg& c) {
    TORCH_CHECK(Q.dim() == 4 && K.dim() == 4, "splash_attention: Q, K, V must be [B, H, N, d]");
    TORCH_CHECK(K.size(0) == Q.size(0) && K.size(1) == Q.size(1) && K.size(3) == Q.size(3),
                "splash_attention: K must be [B, H, NK, d] matching Q");
    asa_params p;
    asa_params_default(&p);
    p.B = (int)Q.size(0);
    p.H = (int)Q.size(1);
    p.NQ = (int)Q.size(2);
    p.NK = (int)K.size(2);
    p.d = (int)Q.size(3);
    p.block_m = (int)c.block_m;
    p.block_n = (int)c.block_n;
    p.k_keep = (int)c.k_keep;
    p.alpha = (float)c.alpha;
    p.sm_scale = (float)c.sm_scale;
    p.causal = c.causal ? 1 : 0;
    p.in_dtype = dtype_code(Q.scalar_type());
    p.out_dtype = c.out_f32 ? ASA_DTYPE_F32 : p.in_dtype;
    p.backend = (int)c.backend;
    p.precision = (int)c.precision;
    p.ref_tile_load = c.ref_tile_load ? 1 : 0;
    p.tau_mode = (int)c.tau_mode;
    p.grad_mode = (int)c.grad_mode;
    return p;
}

at::ScalarType out_type(const asa_params& p) {
    return p.out_dtype == ASA_DTYPE_F32 ? at::kFloat : at::kBFloat16;
}

const void* ptr_or_null(const c10::optional<Tensor>& t) {
    return t.has_value() && t->defined() ? t->data_ptr() : nullptr;
}

void check_positions(const c10::optional<Tensor>& idx, int64_t rows, int64_t n, const char* name,
                     bool causal) {
    if (!causal) return;
    TORCH_CHECK(idx.has_value() && idx->defined(), "splash_attention: ", name,
                " is required when causal=True");
    TORCH_CHECK(idx->scalar_type() == at::kInt && idx->is_contiguous() && idx->numel() == rows * n,
                "splash_attention: ", name, " must be contiguous int32 [B*H, N]");
}

// Per device: pinned host word receiving asynchronous copies of the device
// error word (asa_device_error_async) after each backward and each forward
// with no backward to follow.  A landed non-zero value makes the next call
// raise: no call synchronises, so the report comes one call later.
struct ErrWord {
    std::mutex mu;
    Tensor host[64];
};
ErrWord& err_words() {
    static ErrWord w;
    return w;
}

void raise_pending_error(int dev) {
    ErrWord& w = err_words();
    std::lock_guard<std::mutex> lk(w.mu);
    if (dev < 0 || dev >= 64 || !w.host[dev].defined()) return;
    int* h = w.host[dev].data_ptr<int>();
    const int code = *reinterpret_cast<volatile int*>(h);
    if (code == 0) return;
    *h = 0;
    int cleared = 0;
    asa_device_error((asa_stream_t)c10::cuda::getCurrentCUDAStream(dev).stream(), &cleared);
    check(code, "a previous splash_attention call on this device");
}

void poll_error(int dev) {
    ErrWord& w = err_words();
    std::lock_guard<std::mutex> lk(w.mu);
    if (dev < 0 || dev >= 64) return;
    if (!w.host[dev].defined())
        w.host[dev] = at::zeros({1}, at::TensorOptions().dtype(at::kInt).pinned_memory(true));
    check(asa_device_error_async((asa_stream_t)c10::cuda::getCurrentCUDAStream(dev).stream(),
                                 w.host[dev].data_ptr<int>()),
          "asa_device_error_async");
}

using FwdOut = std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor>;

FwdOut forward_shapes(const Tensor& Q, const Tensor& K, const Cfg& c, bool need_o32,
                      const at::TensorOptions& base) {
    const int64_t B = Q.size(0), H = Q.size(1), NQ = Q.size(2), NK = K.size(2), d = Q.size(3);
    const int64_t BH = B * H;
    const int64_t nqb = (NQ + c.block_m - 1) / c.block_m, nkb = (NK + c.block_n - 1) / c.block_n;
    const auto ot = c.out_f32 ? at::kFloat : Q.scalar_type();
    Tensor O = at::empty({B, H, NQ, d}, base.dtype(ot));
    // fp32 outputs: O itself is the backward's fp32 copy, so O32 stays empty
    // (operator outputs may not alias one another)
    Tensor O32 = at::empty({(need_o32 && ot != at::kFloat) ? B : 0, H, NQ, d},
                           base.dtype(at::kFloat));
    Tensor tau = at::empty({BH, NQ}, base.dtype(at::kFloat));
    Tensor M = at::empty({BH, nqb, nkb}, base.dtype(at::kByte));
    Tensor ptr = at::empty({BH, nqb + 1}, base.dtype(at::kInt));
    Tensor idx = at::empty({BH, nqb * nkb}, base.dtype(at::kInt));
    Tensor rown = at::empty({BH, NQ}, base.dtype(at::kFloat));
    return {O, O32, tau, M, ptr, idx, rown};
}

Cfg cfg_of(double alpha, double sm_scale, int64_t k_keep, int64_t block_m, int64_t block_n,
           bool causal, int64_t backend, int64_t precision, bool out_f32, bool ref_tile_load,
           int64_t tau_mode, int64_t grad_mode) {
    return Cfg{alpha, sm_scale, k_keep, block_m, block_n, causal, backend, precision, out_f32,
               ref_tile_load, tau_mode, grad_mode};
}

FwdOut forward_cuda(const Tensor& Q_, const Tensor& K_, const Tensor& V_,
                    const c10::optional<Tensor>& Qidx, const c10::optional<Tensor>& Kidx,
                    double alpha, double sm_scale, int64_t k_keep, int64_t block_m,
                    int64_t block_n, bool causal, int64_t backend, int64_t precision,
                    bool out_f32, bool ref_tile_load, int64_t tau_mode, int64_t grad_mode,
                    bool fused_forward, bool need_o32) {
    TORCH_CHECK(Q_.is_cuda() && K_.is_cuda() && V_.is_cuda(),
                "splash_attention: tensors must be on a CUDA device");   // reference :543
    TORCH_CHECK(V_.sizes() == K_.sizes() && V_.scalar_type() == Q_.scalar_type() &&
                    K_.scalar_type() == Q_.scalar_type(),
                "splash_attention: V must match K in shape and Q in dtype");
    c10::cuda::CUDAGuard guard(Q_.device());
    const Tensor Q = Q_.contiguous(), K = K_.contiguous(), V = V_.contiguous();
    const Cfg c = cfg_of(alpha, sm_scale, k_keep, block_m, block_n, causal, backend, precision,
                         out_f32, ref_tile_load, tau_mode, grad_mode);
    asa_params p = make_params(Q, K, c);
    p.fused_forward = fused_forward ? 1 : 0;
    check_positions(Qidx, (int64_t)p.B * p.H, p.NQ, "Q_idx", causal);
    check_positions(Kidx, (int64_t)p.B * p.H, p.NK, "K_idx", causal);
    FwdOut out = forward_shapes(Q, K, c, need_o32, Q.options());
    auto& [O, O32, tau, M, ptr, idx, rown] = out;
    size_t fwd = 0, bwd = 0;
    check(asa_workspace_bytes(&p, &fwd, &bwd), "asa_workspace_bytes");
    Tensor ws = at::empty({(int64_t)fwd}, Q.options().dtype(at::kByte));
    const int dev = Q.get_device();
    raise_pending_error(dev);
    auto st = (asa_stream_t)c10::cuda::getCurrentCUDAStream(dev).stream();
    check(asa_forward(&p, Q.data_ptr(), K.data_ptr(), V.data_ptr(),
                      (const int32_t*)ptr_or_null(Qidx), (const int32_t*)ptr_or_null(Kidx),
                      O.data_ptr(),
                      O32.numel() ? O32.data_ptr<float>()
                                  : (O.scalar_type() == at::kFloat ? O.data_ptr<float>() : nullptr),
                      tau.data_ptr<float>(), M.data_ptr<uint8_t>(), ptr.data_ptr<int32_t>(),
                      idx.data_ptr<int32_t>(), rown.data_ptr<float>(), ws.data_ptr(), fwd, st),
          "asa_forward");
    if (!need_o32) poll_error(dev);
    return out;
}

FwdOut forward_meta(const Tensor& Q, const Tensor& K, const Tensor& V,
                    const c10::optional<Tensor>& Qidx, const c10::optional<Tensor>& Kidx,
                    double alpha, double sm_scale, int64_t k_keep, int64_t block_m,
                    int64_t block_n, bool causal, int64_t backend, int64_t precision,
                    bool out_f32, bool ref_tile_load, int64_t tau_mode, int64_t grad_mode,
                    bool fused_forward, bool need_o32) {
    const Cfg c = cfg_of(alpha, sm_scale, k_keep, block_m, block_n, causal, backend, precision,
                         out_f32, ref_tile_load, tau_mode, grad_mode);
    return forward_shapes(Q, K, c, need_o32, Q.options());
}

std::tuple<Tensor, Tensor, Tensor> backward_cuda(
    const Tensor& Q_, const Tensor& K_, const Tensor& V_, const c10::optional<Tensor>& Qidx,
    const c10::optional<Tensor>& Kidx, const Tensor& O32, const Tensor& tau, const Tensor& M,
    const Tensor& csr_ptr, const Tensor& csr_idx, const Tensor& rownorm, const Tensor& dO_,
    double alpha, double sm_scale, int64_t k_keep, int64_t block_m, int64_t block_n, bool causal,
    int64_t backend, int64_t precision, bool out_f32, bool ref_tile_load, int64_t tau_mode,
    int64_t grad_mode) {
    c10::cuda::CUDAGuard guard(Q_.device());
    const Tensor Q = Q_.contiguous(), K = K_.contiguous(), V = V_.contiguous();
    const Tensor dO = dO_.to(Q.scalar_type()).contiguous();
    const Cfg c = cfg_of(alpha, sm_scale, k_keep, block_m, block_n, causal, backend, precision,
                         out_f32, ref_tile_load, tau_mode, grad_mode);
    asa_params p = make_params(Q, K, c);
    TORCH_CHECK(O32.numel() == Q.numel() && O32.scalar_type() == at::kFloat,
                "splash_attention::backward: the forward did not keep its fp32 output");
    const auto ot = out_type(p);
    Tensor dQ = at::empty(Q.sizes(), Q.options().dtype(ot));
    Tensor dK = at::empty(K.sizes(), K.options().dtype(ot));
    Tensor dV = at::empty(K.sizes(), K.options().dtype(ot));
    size_t fwd = 0, bwd = 0;
    check(asa_workspace_bytes(&p, &fwd, &bwd), "asa_workspace_bytes");
    Tensor ws = at::empty({(int64_t)bwd}, Q.options().dtype(at::kByte));
    const int dev = Q.get_device();
    raise_pending_error(dev);
    auto st = (asa_stream_t)c10::cuda::getCurrentCUDAStream(dev).stream();
    check(asa_backward(&p, Q.data_ptr(), K.data_ptr(), V.data_ptr(),
                       (const int32_t*)ptr_or_null(Qidx), (const int32_t*)ptr_or_null(Kidx),
                       O32.data_ptr<float>(), tau.data_ptr<float>(), M.data_ptr<uint8_t>(),
                       csr_ptr.data_ptr<int32_t>(), csr_idx.data_ptr<int32_t>(),
                       rownorm.data_ptr<float>(), dO.data_ptr(), dQ.data_ptr(), dK.data_ptr(),
                       dV.data_ptr(), ws.data_ptr(), bwd, st),
          "asa_backward");
    poll_error(dev);
    return {dQ, dK, dV};
}

std::tuple<Tensor, Tensor, Tensor> backward_meta(
    const Tensor& Q, const Tensor& K, const Tensor& V, const c10::optional<Tensor>& Qidx,
    const c10::optional<Tensor>& Kidx, const Tensor& O32, const Tensor& tau, const Tensor& M,
    const Tensor& csr_ptr, const Tensor& csr_idx, const Tensor& rownorm, const Tensor& dO,
    double alpha, double sm_scale, int64_t k_keep, int64_t block_m, int64_t block_n, bool causal,
    int64_t backend, int64_t precision, bool out_f32, bool ref_tile_load, int64_t tau_mode,
    int64_t grad_mode) {
    const auto ot = out_f32 ? at::kFloat : Q.scalar_type();
    return {at::empty(Q.sizes(), Q.options().dtype(ot)), at::empty(K.sizes(), K.options().dtype(ot)),
            at::empty(K.sizes(), K.options().dtype(ot))};
}

}  // namespace

TORCH_LIBRARY(splash_attention, m) {
    m.def(
        "forward(Tensor Q, Tensor K, Tensor V, Tensor? Q_idx, Tensor? K_idx, float alpha, "
        "float sm_scale, int k_keep, int block_m, int block_n, bool causal, int backend, "
        "int precision, bool out_f32, bool ref_tile_load, int tau_mode, int grad_mode, "
        "bool fused_forward, bool need_o32) -> "
        "(Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor)");
    m.def(
        "backward(Tensor Q, Tensor K, Tensor V, Tensor? Q_idx, Tensor? K_idx, Tensor O32, "
        "Tensor tau, Tensor M, Tensor csr_ptr, Tensor csr_idx, Tensor rownorm, Tensor dO, "
        "float alpha, float sm_scale, int k_keep, int block_m, int block_n, bool causal, "
        "int backend, int precision, bool out_f32, bool ref_tile_load, int tau_mode, int grad_mode) "
        "-> (Tensor, Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(splash_attention, CUDA, m) {
    m.impl("forward", &forward_cuda);
    m.impl("backward", &backward_cuda);
}

TORCH_LIBRARY_IMPL(splash_attention, Meta, m) {
    m.impl("forward", &forward_meta);
    m.impl("backward", &backward_meta);
}
