// y = x @ w^T with a fused epilogue.  float32 operands run on CUDA cores (the SDM_F32 precision mode: exact
// float32 products, float32 accumulation in k order); bfloat16 operands run on the tensor cores: tcgen05
// (gemm_tc.cu) for tile-sized row counts, mma.sync below for decode-sized ones (at most 32 rows).
#include "kernels.cuh"

namespace sdm {

constexpr int SG_BM = 128, SG_BN = 64, SG_BK = 16;

template <typename TA, typename Epi>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const TA* __restrict__ x, int64_t ldx,
                                                        const TA* __restrict__ w, int64_t ldw, int64_t rows, int K,
                                                        int n, Epi epi, int kwrap) {
  pdl_enter();
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
  return launch_k(gemm_simt_kernel<TA, Epi>, dim3(grid), dim3(256), 0, st, x, ldx, w, ldw, rows, K, n, epi, kwrap);
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
  pdl_enter();
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
  return launch_k(kern, dim3((unsigned)grid), dim3(SK_WARPS * 32), smem, st, x, ldx, w, ldw, (int)rows, K, n, epi,
                  kwrap);
}

// ------------------------------------------------------------------------------------- small-M tensor-core GEMM
// Decode-sized bf16 products (at most SMT_MAX_ROWS rows) on the tensor cores with mma.sync m16n8k16 (bf16 operands,
// float32 accumulation: the products and accumulation precision of the tcgen05 path).  A CTA owns 8 output columns of
// one 32-row block (blockIdx.y; the weight columns stay L2-resident across the row blocks, so a few hundred decode
// streams keep every SM busy where a 256-wide tensor-core tile would occupy a handful); its 8 warps split the K
// range in 64-wide blocks (a K wrap, x = [hi | lo] against one w, is just more blocks reading the
// same weights), each warp covering all rows as two 16-row tiles; the 8 partial 32 x 8 tiles are summed in shared
// memory in warp order, so results are deterministic.  Inside a 64-block thread t of a quad holds 16 consecutive k
// of its A rows and B column (two 16-byte loads each) and feeds them to four k-steps: slots (2t, 2t+1, 2t+8, 2t+9)
// of step s carry its values 4s .. 4s+3 -- the same permutation of k for A and B, so the dot products are unchanged.
constexpr int SMT_WARPS = 8;
constexpr int64_t SMT_MAX_ROWS = 512;

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t u4w(const uint4& u, int i) {
  return i == 0 ? u.x : (i == 1 ? u.y : (i == 2 ? u.z : u.w));
}

template <typename Epi>
__global__ void __launch_bounds__(SMT_WARPS * 32) gemm_small_tc_kernel(const bf16_t* __restrict__ x, int64_t ldx,
                                                                      const bf16_t* __restrict__ w, int64_t ldw,
                                                                      int rows, int K, int n, Epi epi, int kwrap) {
  pdl_enter();
  __shared__ float part[SMT_WARPS][32][9];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row0 = blockIdx.y * 32;
  x += (int64_t)row0 * ldx;
  rows -= row0;
  const int g = lane >> 2, t = lane & 3;
  const int n0 = blockIdx.x * 8;
  const int nb = n0 + g;  // this thread's B column
  const bf16_t* wrow = w + (int64_t)(nb < n ? nb : n - 1) * ldw;
  float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
  for (int kb = warp; kb < K / 64; kb += SMT_WARPS) {
    const int k = kb * 64 + 16 * t, kw = k % kwrap;
    const uint4 b0 = nb < n ? *reinterpret_cast<const uint4*>(wrow + kw) : z4;
    const uint4 b1 = nb < n ? *reinterpret_cast<const uint4*>(wrow + kw + 8) : z4;
    uint4 a[2][2][2];  // [row tile][row g | g + 8][k 0-7 | 8-15]
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int rh = 0; rh < 2; ++rh) {
        const int row = mt * 16 + rh * 8 + g;
        const bf16_t* xr = x + (int64_t)row * ldx + k;
        a[mt][rh][0] = row < rows ? *reinterpret_cast<const uint4*>(xr) : z4;
        a[mt][rh][1] = row < rows ? *reinterpret_cast<const uint4*>(xr + 8) : z4;
      }
#pragma unroll
    for (int s4 = 0; s4 < 4; ++s4) {
      const int h = s4 >> 1, wi = (s4 & 1) * 2;  // values 4*s4 .. 4*s4+3 are words wi, wi+1 of chunk h
      const uint32_t bw0 = u4w(h ? b1 : b0, wi), bw1 = u4w(h ? b1 : b0, wi + 1);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
        mma_bf16_16816(c[mt], u4w(a[mt][0][h], wi), u4w(a[mt][1][h], wi), u4w(a[mt][0][h], wi + 1),
                       u4w(a[mt][1][h], wi + 1), bw0, bw1);
    }
  }
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    part[warp][mt * 16 + g][2 * t] = c[mt][0];
    part[warp][mt * 16 + g][2 * t + 1] = c[mt][1];
    part[warp][mt * 16 + g + 8][2 * t] = c[mt][2];
    part[warp][mt * 16 + g + 8][2 * t + 1] = c[mt][3];
  }
  __syncthreads();
  const int row = tid >> 3, cc = tid & 7, col = n0 + cc;
  float v = 0.f;
#pragma unroll
  for (int q = 0; q < SMT_WARPS; ++q) v += part[q][row][cc];
  if (row < rows && col < n) epi.apply(row0 + row, col, v);
}

// The same product with a 32 x 32 output tile per CTA (n >= 32): each CTA reads its 32 rows of x once for 32 columns
// instead of 8, a quarter of the x traffic from L2, which bounds the 8-column tiles at a few hundred rows.  The
// eight warps split K in 32-wide blocks (warp w takes blocks w, w + 8, ...); inside a block thread t of a quad
// holds 8 consecutive k of its A rows and of its four B columns (one 16-byte load each) and feeds them to two k-steps
// (values 4s .. 4s+3 of step s, the same permutation for A and B); 2 x 4 accumulator tiles per warp, the 8 partial
// 32 x 32 tiles summed in shared memory in warp order (deterministic).
template <typename Epi>
__global__ void __launch_bounds__(SMT_WARPS * 32) gemm_small_tc32_kernel(const bf16_t* __restrict__ x, int64_t ldx,
                                                                        const bf16_t* __restrict__ w, int64_t ldw,
                                                                        int rows, int K, int n, Epi epi, int kwrap) {
  pdl_enter();
  __shared__ float part[SMT_WARPS][32][33];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row0 = blockIdx.y * 32;
  x += (int64_t)row0 * ldx;
  rows -= row0;
  const int g = lane >> 2, t = lane & 3;
  const int n0 = blockIdx.x * 32;
  const bf16_t* wrow[4];
  bool bval[4];
#pragma unroll
  for (int ct = 0; ct < 4; ++ct) {
    const int nb = n0 + ct * 8 + g;  // this thread's B column of column tile ct
    bval[ct] = nb < n;
    wrow[ct] = w + (int64_t)(nb < n ? nb : n - 1) * ldw;
  }
  float c[2][4][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int ct = 0; ct < 4; ++ct)
#pragma unroll
      for (int e = 0; e < 4; ++e) c[mt][ct][e] = 0.f;
  const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
  for (int kb = warp; kb < K / 32; kb += SMT_WARPS) {
    const int k = kb * 32 + 8 * t, kw = k % kwrap;
    uint4 b[4], a[2][2];  // a: [row tile][row g | g + 8]
#pragma unroll
    for (int ct = 0; ct < 4; ++ct) b[ct] = bval[ct] ? *reinterpret_cast<const uint4*>(wrow[ct] + kw) : z4;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int rh = 0; rh < 2; ++rh) {
        const int row = mt * 16 + rh * 8 + g;
        a[mt][rh] = row < rows ? *reinterpret_cast<const uint4*>(x + (int64_t)row * ldx + k) : z4;
      }
#pragma unroll
    for (int s2 = 0; s2 < 2; ++s2)
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int ct = 0; ct < 4; ++ct)
          mma_bf16_16816(c[mt][ct], u4w(a[mt][0], 2 * s2), u4w(a[mt][1], 2 * s2), u4w(a[mt][0], 2 * s2 + 1),
                         u4w(a[mt][1], 2 * s2 + 1), u4w(b[ct], 2 * s2), u4w(b[ct], 2 * s2 + 1));
  }
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int ct = 0; ct < 4; ++ct) {
      part[warp][mt * 16 + g][ct * 8 + 2 * t] = c[mt][ct][0];
      part[warp][mt * 16 + g][ct * 8 + 2 * t + 1] = c[mt][ct][1];
      part[warp][mt * 16 + g + 8][ct * 8 + 2 * t] = c[mt][ct][2];
      part[warp][mt * 16 + g + 8][ct * 8 + 2 * t + 1] = c[mt][ct][3];
    }
  __syncthreads();
  for (int o = tid; o < 32 * 32; o += SMT_WARPS * 32) {
    const int row = o >> 5, cc = o & 31, col = n0 + cc;
    float v = 0.f;
#pragma unroll
    for (int q = 0; q < SMT_WARPS; ++q) v += part[q][row][cc];
    if (row < rows && col < n) epi.apply(row0 + row, col, v);
  }
}

static bool small_tc_ok(const bf16_t* x, int64_t ldx, const bf16_t* w, int64_t ldw, int64_t rows, int K, int kwrap) {
  const uintptr_t ax = reinterpret_cast<uintptr_t>(x), aw = reinterpret_cast<uintptr_t>(w);
  return rows >= 1 && rows <= SMT_MAX_ROWS && K % 64 == 0 && kwrap % 64 == 0 && ldx % 8 == 0 && ldw % 8 == 0 &&
         ax % 16 == 0 && aw % 16 == 0;
}

template <typename TA, typename Epi>
cudaError_t launch_gemm(const TA* x, int64_t ldx, const TA* w, int64_t ldw, int64_t rows, int K, int n, Epi epi,
                        cudaStream_t st, int kwrap) {
  if (kwrap <= 0) kwrap = K;
  if (K % kwrap) return cudaErrorInvalidValue;
  if (rows == 0 || n == 0) return cudaSuccess;
  if constexpr (sizeof(TA) == 2) {
    if (small_tc_ok(x, ldx, w, ldw, rows, K, kwrap)) {
      LaunchScope scope_("gemm_small_tc", st);
      // 32-column tiles when they still give every SM a CTA (a few hundred rows), else 8-column tiles
      if (n >= 32 && K % 32 == 0 && kwrap % 32 == 0 && ceil_div(n, 32) * ceil_div(rows, 32) >= 148)
        return launch_k(gemm_small_tc32_kernel<Epi>, dim3((unsigned)ceil_div(n, 32), (unsigned)ceil_div(rows, 32)),
                        dim3(SMT_WARPS * 32), 0, st, x, ldx, w, ldw, (int)rows, K, n, epi, kwrap);
      return launch_k(gemm_small_tc_kernel<Epi>, dim3((unsigned)ceil_div(n, 8), (unsigned)ceil_div(rows, 32)),
                      dim3(SMT_WARPS * 32), 0, st, x, ldx, w, ldw, (int)rows, K, n, epi, kwrap);
    }
  }
  if (skinny_ok(x, ldx, w, ldw, rows, K, kwrap))
    return launch_gemm_skinny<TA, Epi>(x, ldx, w, ldw, rows, K, n, epi, st, kwrap);
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
