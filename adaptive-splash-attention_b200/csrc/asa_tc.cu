// asa_tc.cu -- tcgen05 / TMEM / TMA kernels (bf16, d in {64,128}, 128x128 tiles).
#include "asa_internal.h"

namespace asa {

bool tc_supported(const Shape& s) { (void)s; return false; }
size_t tc_fwd_workspace(const Shape&) { return 0; }
size_t tc_bwd_workspace(const Shape&) { return 0; }
cudaError_t tc_tau_mask(const Shape&, const void*, const void*, const int32_t*, const int32_t*,
                        float*, uint8_t*, void*, int*, cudaStream_t) {
    return cudaErrorNotSupported;
}
cudaError_t tc_forward(const Shape&, const void*, const void*, const void*, const int32_t*,
                       const int32_t*, const float*, const int32_t*, const int32_t*, void*, float*,
                       float*, void*, int*, cudaStream_t) {
    return cudaErrorNotSupported;
}
cudaError_t tc_backward(const Shape&, const void*, const void*, const void*, const int32_t*,
                        const int32_t*, const float*, const float*, const int32_t*,
                        const int32_t*, const int32_t*, const int32_t*, const float*, const void*,
                        void*, void*, void*, void*, int*, cudaStream_t) {
    return cudaErrorNotSupported;
}

}  // namespace asa
