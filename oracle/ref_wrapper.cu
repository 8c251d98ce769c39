// ref_wrapper.cu -- compiles the reference's own CUDA source
// (source/adasplashattention.cu, included unmodified from the reference
// checkout via -I) into a loadable module, for generating golden vectors.
//
// TEST INFRASTRUCTURE ONLY (oracle/).  Two adaptations, neither touching the
// reference's arithmetic:
//  * adasplashattention.cu:554 and :629 put `#BLOCK_M` inside a TORCH_CHECK
//    message, which does not compile.  TORCH_CHECK is redefined below as a
//    macro that drops its message arguments, so the stray token vanishes in
//    preprocessing.
//  * the reference exports only forward/backward (:702-705), so τ and the
//    block mask are not observable.  ref_mask_tau() below launches the
//    reference's own build_mask_kernel and build_lookup_kernel exactly as
//    forward_splash does (:558-591) and returns their outputs.
#include <torch/extension.h>
#include <stdexcept>
#undef TORCH_CHECK
#define TORCH_CHECK(cond, ...)                                                  \
    do {                                                                        \
        if (!(cond)) throw std::runtime_error("reference check failed: " #cond); \
    } while (0)

#include "adasplashattention.cu"

std::vector<torch::Tensor> ref_mask_tau(torch::Tensor Q, torch::Tensor K, torch::Tensor Q_idx,
                                        torch::Tensor K_idx, double sm_scale_d, double alpha_d) {
    float sm_scale = (float)sm_scale_d;
    float alpha = std::max(1.05f, std::min((float)alpha_d, 3.0f));
    auto d = Q.size(3);
    auto B = Q.size(0), H = Q.size(1), NQ = Q.size(2), NK = K.size(2);
    int nQB = (NQ + BLOCK_M - 1) / BLOCK_M;
    int nKB = (NK + BLOCK_N - 1) / BLOCK_N;
    auto opts8 = torch::TensorOptions().dtype(torch::kInt8).device(Q.device());
    auto optsF = torch::TensorOptions().dtype(Q.dtype()).device(Q.device());
    auto M = torch::zeros({B * H, nQB, nKB}, opts8);
    auto taus = torch::zeros({B * H, NQ}, optsF);
    auto Qi_ptr = torch::zeros({B * H, nQB + 1}, torch::dtype(torch::kInt32).device(Q.device()));
    auto Qi_idx = torch::zeros({B * H, nQB * nKB}, torch::dtype(torch::kInt32).device(Q.device()));
    dim3 grid1(nQB, B * H);
    build_mask_kernel<<<grid1, BLOCK_M, BLOCK_N * d * sizeof(float)>>>(
        Q.data_ptr<float>(), K.data_ptr<float>(), Q_idx.data_ptr<int>(), K_idx.data_ptr<int>(),
        B, H, NQ, NK, d, alpha, sm_scale, M.data_ptr<int8_t>(), taus.data_ptr<float>(), nQB, nKB);
    CUDA_CHECK(cudaGetLastError());
    build_lookup_kernel<<<B * H, 32>>>(M.data_ptr<int8_t>(), B, H, nQB, nKB,
                                       Qi_ptr.data_ptr<int32_t>(), Qi_idx.data_ptr<int32_t>());
    CUDA_CHECK(cudaGetLastError());
    CUDA_CHECK(cudaDeviceSynchronize());
    return {taus, M, Qi_ptr, Qi_idx};
}

TORCH_LIBRARY(REF_OPS_NS, m) {
    m.def("mask_tau", &ref_mask_tau);
}
