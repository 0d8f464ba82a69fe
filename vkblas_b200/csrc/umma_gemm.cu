// umma_gemm.cu -- tcgen05 GEMM (placeholder until the tensor-core kernels land).
#include "common.cuh"

namespace vkb {
bool umma_supported(const GemmProblem&) { return false; }
cudaError_t launch_umma_gemm(const GemmProblem&, int, int*, cudaStream_t) {
    return cudaErrorNotSupported;
}
}  // namespace vkb
