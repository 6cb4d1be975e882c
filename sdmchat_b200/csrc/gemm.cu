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

// ---------------------------------------------------------------------------------------------- skinny GEMM
// Decode-sized products (at most 32 rows): the tile GEMMs would keep only a handful of SMs busy, so here every warp
// owns one output column.  The rows are staged once per CTA in shared memory as float32, K_eff = kwrap columns at a
// time (up to SK_KC): with a K wrap (x = [hi | lo] against one w) the copies are added as they are staged, which is
// exact for a bf16 hi/lo split and leaves one product per weight.  A warp streams its weight row (16 bytes per lane
// per step, coalesced), accumulates all rows' partial dot products in registers, and a 31-shuffle reduce-scatter
// butterfly leaves row m's sum in lane m, which applies the epilogue.
constexpr int SK_WARPS = 8;
constexpr int SK_MAX_ROWS = 32;
constexpr int SK_KC = 1024;  // staged columns per pass (32 rows x 1024 x 4 B = 128 KB)

template <typename TA>
struct Vec8 {
  float v[8];
};
__device__ __forceinline__ Vec8<bf16_t> load8(const bf16_t* p) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
  Vec8<bf16_t> r;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    r.v[2 * i] = f.x;
    r.v[2 * i + 1] = f.y;
  }
  return r;
}
__device__ __forceinline__ Vec8<float> load8(const float* p) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  return {{a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w}};
}

template <typename TA, typename Epi>
__global__ void __launch_bounds__(SK_WARPS * 32) gemm_skinny_kernel(const TA* __restrict__ x, int64_t ldx,
                                                                   const TA* __restrict__ w, int64_t ldw, int rows,
                                                                   int K, int n, Epi epi, int kwrap) {
  extern __shared__ __align__(16) unsigned char sk_smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int col = blockIdx.x * SK_WARPS + warp;
  const int copies = K / kwrap;
  float* xs = reinterpret_cast<float*>(sk_smem);  // (rows, kc) float32
  float acc[SK_MAX_ROWS];
#pragma unroll
  for (int m = 0; m < SK_MAX_ROWS; ++m) acc[m] = 0.f;
  const TA* wr = w + (int64_t)(col < n ? col : 0) * ldw;
  for (int k0 = 0; k0 < kwrap; k0 += SK_KC) {
    const int kc = min(SK_KC, kwrap - k0);
    const int vpr = kc / 8;  // 8-column vectors per row
    __syncthreads();          // the previous pass's reads of xs are done
    for (int i = tid; i < rows * vpr; i += SK_WARPS * 32) {
      const int r = i / vpr, c = (i - r * vpr) * 8;
      Vec8<TA> v = load8(x + (int64_t)r * ldx + k0 + c);
      for (int cp = 1; cp < copies; ++cp) {
        const Vec8<TA> u = load8(x + (int64_t)r * ldx + (int64_t)cp * kwrap + k0 + c);
#pragma unroll
        for (int e = 0; e < 8; ++e) v.v[e] += u.v[e];
      }
      float4* d = reinterpret_cast<float4*>(xs + (int64_t)r * kc + c);
      d[0] = make_float4(v.v[0], v.v[1], v.v[2], v.v[3]);
      d[1] = make_float4(v.v[4], v.v[5], v.v[6], v.v[7]);
    }
    __syncthreads();
    if (col < n) {
      for (int kk = lane * 8; kk < kc; kk += 256) {
        const Vec8<TA> wv = load8(wr + k0 + kk);
#pragma unroll
        for (int m = 0; m < SK_MAX_ROWS; ++m) {
          if (m < rows) {
            const float4 a = *reinterpret_cast<const float4*>(xs + (int64_t)m * kc + kk);
            const float4 b = *reinterpret_cast<const float4*>(xs + (int64_t)m * kc + kk + 4);
            acc[m] = fmaf(a.x, wv.v[0], acc[m]);
            acc[m] = fmaf(a.y, wv.v[1], acc[m]);
            acc[m] = fmaf(a.z, wv.v[2], acc[m]);
            acc[m] = fmaf(a.w, wv.v[3], acc[m]);
            acc[m] = fmaf(b.x, wv.v[4], acc[m]);
            acc[m] = fmaf(b.y, wv.v[5], acc[m]);
            acc[m] = fmaf(b.z, wv.v[6], acc[m]);
            acc[m] = fmaf(b.w, wv.v[7], acc[m]);
          }
        }
      }
    }
  }
  if (col >= n) return;
  // reduce-scatter: after the step of width o, this lane keeps the rows whose bit matches its lane bit
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float mine = upper ? acc[i + o] : acc[i];
      const float other = upper ? acc[i] : acc[i + o];
      acc[i] = mine + __shfl_xor_sync(0xffffffffu, other, o);
    }
  }
  if (lane < rows) epi.apply(lane, col, acc[0]);
}

template <typename TA>
static bool skinny_ok(const TA* x, int64_t ldx, const TA* w, int64_t ldw, int64_t rows, int K, int kwrap) {
  const uintptr_t ax = reinterpret_cast<uintptr_t>(x), aw = reinterpret_cast<uintptr_t>(w);
  return rows >= 1 && rows <= SK_MAX_ROWS && K % 8 == 0 && kwrap % 8 == 0 && ldx % 8 == 0 && ldw % 8 == 0 &&
         ax % 16 == 0 && aw % 16 == 0;
}

template <typename TA, typename Epi>
static cudaError_t launch_gemm_skinny(const TA* x, int64_t ldx, const TA* w, int64_t ldw, int64_t rows, int K, int n,
                                     Epi epi, cudaStream_t st, int kwrap) {
  const size_t smem = (size_t)rows * (kwrap < SK_KC ? kwrap : SK_KC) * sizeof(float);
  auto kern = gemm_skinny_kernel<TA, Epi>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int64_t grid = ceil_div(n, SK_WARPS);
  LaunchScope scope_("gemm_skinny", st);
  kern<<<(unsigned)grid, SK_WARPS * 32, smem, st>>>(x, ldx, w, ldw, (int)rows, K, n, epi, kwrap);
  return cudaGetLastError();
}

template <typename TA, typename Epi>
cudaError_t launch_gemm(const TA* x, int64_t ldx, const TA* w, int64_t ldw, int64_t rows, int K, int n, Epi epi,
                        cudaStream_t st, int kwrap) {
  if (kwrap <= 0) kwrap = K;
  if (K % kwrap) return cudaErrorInvalidValue;
  if (rows == 0 || n == 0) return cudaSuccess;
  if (skinny_ok(x, ldx, w, ldw, rows, K, kwrap)) return launch_gemm_skinny<TA, Epi>(x, ldx, w, ldw, rows, K, n, epi, st, kwrap);
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
