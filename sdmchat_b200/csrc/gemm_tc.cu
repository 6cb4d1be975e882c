// placeholder: replaced by the tcgen05 GEMM
#include "kernels.cuh"
namespace sdm {
bool tc_gemm_supported(const void*, int64_t, const void*, int64_t, int) { return false; }
template <typename Epi>
cudaError_t launch_gemm_tc(const bf16_t*, int64_t, const bf16_t*, int64_t, int64_t, int, int, Epi, cudaStream_t) {
  return cudaErrorNotSupported;
}
template cudaError_t launch_gemm_tc<EpiF32>(const bf16_t*, int64_t, const bf16_t*, int64_t, int64_t, int, int, EpiF32, cudaStream_t);
template cudaError_t launch_gemm_tc<EpiProj>(const bf16_t*, int64_t, const bf16_t*, int64_t, int64_t, int, int, EpiProj, cudaStream_t);
template cudaError_t launch_gemm_tc<EpiStore<bf16_t>>(const bf16_t*, int64_t, const bf16_t*, int64_t, int64_t, int, int, EpiStore<bf16_t>, cudaStream_t);
template cudaError_t launch_gemm_tc<EpiF32R<bf16_t>>(const bf16_t*, int64_t, const bf16_t*, int64_t, int64_t, int, int, EpiF32R<bf16_t>, cudaStream_t);
template cudaError_t launch_gemm_tc<EpiResid<bf16_t>>(const bf16_t*, int64_t, const bf16_t*, int64_t, int64_t, int, int, EpiResid<bf16_t>, cudaStream_t);
}
