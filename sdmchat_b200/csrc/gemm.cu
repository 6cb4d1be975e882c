// y = x @ w^T with a fused epilogue.  float32 operands run on CUDA cores (the SDM_F32 precision mode: exact
// float32 products, float32 accumulation in k order); bfloat16 operands run on the tcgen05 tensor cores
// (gemm_tc.cu) whenever the shape allows it.
#include "kernels.cuh"

namespace sdm {

constexpr int SG_BM = 128, SG_BN = 64, SG_BK = 16;

template <typename TA, typename Epi>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const TA* __restrict__ x, int64_t ldx,
                                                        const TA* __restrict__ w, int64_t ldw, int64_t rows, int K,
                                                        int n, Epi epi, int kwrap) {
  __shared__ float As[SG_BK][SG_BM + 4];
  __shared__ float Bs[SG_BK][SG_BN + 4];
  const int tid = threadIdx.x;
  const int tx = tid % 16, ty = tid / 16;
  const int64_t row0 = (int64_t)blockIdx.y * SG_BM;
  const int col0 = blockIdx.x * SG_BN;
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  for (int k0 = 0; k0 < K; k0 += SG_BK) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int idx = tid + q * 256;
      const int m = idx / SG_BK, kk = idx % SG_BK;
      const int64_t r = row0 + m;
      const int kg = k0 + kk;
      As[kk][m] = (r < rows && kg < K) ? to_f32(x[r * ldx + kg]) : 0.f;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int idx = tid + q * 256;
      const int nn = idx / SG_BK, kk = idx % SG_BK;
      const int c = col0 + nn;
      const int kg = k0 + kk;
      Bs[kk][nn] = (c < n && kg < K) ? to_f32(w[(int64_t)c * ldw + (kg % kwrap)]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SG_BK; ++kk) {
      float av[8], bv[4];
#pragma unroll
      for (int i = 0; i < 8; ++i) av[i] = As[kk][ty * 8 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t r = row0 + ty * 8 + i;
    if (r >= rows) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = col0 + tx * 4 + j;
      if (c < n) epi.apply(r, c, acc[i][j]);
    }
  }
}

template <typename TA, typename Epi>
cudaError_t launch_gemm_simt(const TA* x, int64_t ldx, const TA* w, int64_t ldw, int64_t rows, int K, int n, Epi epi,
                             cudaStream_t st, int kwrap) {
  if (rows == 0 || n == 0) return cudaSuccess;
  dim3 grid((unsigned)ceil_div(n, SG_BN), (unsigned)ceil_div(rows, SG_BM));
  LaunchScope scope_("gemm_simt", st);
  gemm_simt_kernel<TA, Epi><<<grid, 256, 0, st>>>(x, ldx, w, ldw, rows, K, n, epi, kwrap);
  return cudaGetLastError();
}

template <typename TA, typename Epi>
cudaError_t launch_gemm(const TA* x, int64_t ldx, const TA* w, int64_t ldw, int64_t rows, int K, int n, Epi epi,
                        cudaStream_t st, int kwrap) {
  if (kwrap <= 0) kwrap = K;
  if (K % kwrap) return cudaErrorInvalidValue;
  if constexpr (sizeof(TA) == 2) {
    if (tc_gemm_supported(x, ldx, w, ldw, K, kwrap))
      return launch_gemm_tc<Epi>(x, ldx, w, ldw, rows, K, n, epi, st, kwrap);
  }
  return launch_gemm_simt<TA, Epi>(x, ldx, w, ldw, rows, K, n, epi, st, kwrap);
}

#define SDM_GEMM_INST(TA, EPI)                                                                                 \
  template cudaError_t launch_gemm<TA, EPI>(const TA*, int64_t, const TA*, int64_t, int64_t, int, int, EPI, \
                                            cudaStream_t, int);
SDM_GEMM_INST(float, EpiF32)
SDM_GEMM_INST(bf16_t, EpiF32)
SDM_GEMM_INST(float, EpiProj)
SDM_GEMM_INST(bf16_t, EpiProj)
SDM_GEMM_INST(float, EpiStore<float>)
SDM_GEMM_INST(bf16_t, EpiStore<bf16_t>)
SDM_GEMM_INST(float, EpiF32R<float>)
SDM_GEMM_INST(bf16_t, EpiF32R<bf16_t>)
SDM_GEMM_INST(float, EpiResid<float>)
SDM_GEMM_INST(bf16_t, EpiResid<bf16_t>)

}  // namespace sdm
