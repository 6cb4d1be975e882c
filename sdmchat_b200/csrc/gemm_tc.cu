// bfloat16 GEMM on the sm_100a tensor cores: y = x @ w^T with a fused epilogue (tcgen05.mma, TMA, TMEM).
//
// Persistent kernel, one CTA per SM, CTA tile 128 x 128, K step 64 (one 128-byte swizzle atom of bf16 per row).
// Warp roles:
//   warp 0      TMA producer: one lane streams A (x rows) and B (w rows) tiles into a 4-stage ring with
//               cp.async.bulk.tensor, completing on the stage's `full` mbarrier.
//   warp 1      MMA issuer: allocates two 128-column TMEM accumulators; one lane issues 4 tcgen05.mma (K = 16
//               each) per stage from shared-memory descriptors, releases the stage with tcgen05.commit on `empty`
//               and, after a tile's last stage, commits that accumulator's `acc_full` barrier.
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns at a time (warp w reads TMEM lanes 32*(w%4)..+31, i.e.
//               accumulator rows), then hands the accumulator back (`acc_empty`), so tile i's epilogue runs while
//               tile i+1's MMAs fill the other accumulator.
// Epilogues: element-wise ones (Epi::kRowMode false) go through a padded shared-memory transpose so a warp's global
// accesses are 32 consecutive columns of one row; row-owned ones (kRowMode true: the tied-head loss / argmax)
// reduce each thread's row of the tile in registers and write one partial per (row, column tile).
// Every mbarrier wait is bounded (about 4 s of %globaltimer); a wait that gives up sets g_tc_timeout, every role
// falls through to the common exit, and the TMEM columns are released.  No load here reads another GPU's memory
// and none is issued to more than one CTA.
#include <cuda.h>
#include "kernels.cuh"

namespace sdm {

__device__ int g_tc_timeout;

namespace tc {

constexpr int BM = 128, BN = 128, BK = 64, STAGES = 4, THREADS = 192;
constexpr uint32_t A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int STAGE_LD = 33;  // padded row of the epilogue transpose
constexpr size_t RING_BYTES = STAGES * STAGE_BYTES;
constexpr size_t SMEM_BYTES = RING_BYTES + 4 * 32 * STAGE_LD * 4 + 1024;
constexpr uint32_t TMEM_COLS = 2 * BN;

// Instruction descriptor of tcgen05.mma kind::f16: D float32, A and B bfloat16, both K-major, M = 128, N = BN.
constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase with the given parity to complete; false (and the timeout flag set) after ~4 s.
__device__ __noinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > 4000000000ull) {
      atomicExch(&g_tc_timeout, 1);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(const CUtensorMap* map, uint64_t* bar, void* dst, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128 B, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused by swizzled K-major layouts)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;             // descriptor version of sm_100
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(IDESC), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <typename Epi>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int64_t rows,
                   int K, int n, Epi epi, int kwrap) {
  extern __shared__ __align__(1024) unsigned char dsmem[];
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ uint32_t tmem_slot;

  unsigned char* ring = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~(uintptr_t)1023);
  float* stage_all = reinterpret_cast<float*>(ring + RING_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt_count = (K + BK - 1) / BK;
  const int tiles_n = (n + BN - 1) / BN;
  const int64_t tiles = (int64_t)tiles_n * ((rows + BM - 1) / BM);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);  // one arrival per epilogue warp
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int n0 = (int)(t % tiles_n) * BN;
        const int m0 = (int)(t / tiles_n) * BM;
        for (int kt = 0; kt < kt_count; ++kt, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(&empty_bar[s], ph ^ 1u)) {
            ok = false;
            break;
          }
          unsigned char* a_dst = ring + s * STAGE_BYTES;
          mbar_arrive_expect_tx(&full_bar[s], STAGE_BYTES);
          tma_load_2d(&tmA, &full_bar[s], a_dst, kt * BK, m0);
          tma_load_2d(&tmB, &full_bar[s], a_dst + A_BYTES, (kt * BK) % kwrap, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t it = 0, tl = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++tl) {
        const uint32_t buf = tl & 1u, use = tl >> 1;
        if (!mbar_wait(&acc_empty[buf], (use & 1u) ^ 1u)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t dt = tmem + buf * BN;
        for (int kt = 0; kt < kt_count; ++kt, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(&full_bar[s], ph)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a_base = smem_u32(ring + s * STAGE_BYTES);
          const uint32_t b_base = a_base + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_bf16(dt, sw128_desc(a_base + kk * 32), sw128_desc(b_base + kk * 32), (kt | kk) != 0);
          umma_commit(&empty_bar[s]);
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
    }
  } else {
    // epilogue warps 2..5: TMEM lane quarter = warp % 4
    const int q = warp & 3;
    float* stage = stage_all + q * 32 * STAGE_LD;
    uint32_t tl = 0;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++tl) {
      const uint32_t buf = tl & 1u, use = tl >> 1;
      const int tn = (int)(t % tiles_n);
      const int n0 = tn * BN;
      const int64_t m0 = (t / tiles_n) * BM;
      if (!mbar_wait(&acc_full[buf], use & 1u)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int64_t row0 = m0 + q * 32;
      if constexpr (Epi::kRowMode) {
        typename Epi::RowState rs;
        epi.row_begin(rs, row0 + lane, rows, n0);
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(tmem + buf * BN + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, r);
          epi.row_chunk(rs, n0 + c0, n, r);
        }
        epi.row_end(rs, row0 + lane, rows, tn, tiles_n);
      } else {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(tmem + buf * BN + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, r);
#pragma unroll
          for (int j = 0; j < 32; ++j) stage[lane * STAGE_LD + j] = __uint_as_float(r[j]);
          __syncwarp();
          const int col = n0 + c0 + lane;
          const bool col_ok = col < n;
          const typename Epi::Col cc = col_ok ? epi.column(col) : typename Epi::Col{};
          float in[32];
          if constexpr (Epi::kHasInput) {
#pragma unroll
            for (int rr = 0; rr < 32; ++rr)  // all 32 loads in flight before the first use
              in[rr] = (col_ok && row0 + rr < rows) ? epi.load_input(row0 + rr, col) : 0.f;
          }
#pragma unroll 8
          for (int rr = 0; rr < 32; ++rr) {
            const int64_t row = row0 + rr;
            if (row < rows && col_ok)
              epi.store(row, col, stage[rr * STAGE_LD + lane], cc, Epi::kHasInput ? in[rr] : 0.f);
          }
          __syncwarp();
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D bf16 tensor map over a row-major (outer, inner) matrix with row stride ld elements; box (box_outer, 64).
static bool make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, box_outer};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = v > 0 ? v : 148;
  }
  return cached[dev];
}

}  // namespace tc

bool tc_gemm_supported(const void* x, int64_t ldx, const void* w, int64_t ldw, int K, int kwrap) {
  const uintptr_t ax = reinterpret_cast<uintptr_t>(x), aw = reinterpret_cast<uintptr_t>(w);
  const bool wrap_ok = kwrap == K || (kwrap % tc::BK) == 0;  // a wrapped B restarts on a K-step boundary
  return K >= 16 && (K % 8) == 0 && wrap_ok && (ax % 16) == 0 && (aw % 16) == 0 && (ldx % 8) == 0 &&
         (ldw % 8) == 0 && tc::encode_fn() != nullptr;
}

template <typename Epi>
cudaError_t launch_gemm_tc(const bf16_t* x, int64_t ldx, const bf16_t* w, int64_t ldw, int64_t rows, int K, int n,
                           Epi epi, cudaStream_t st, int kwrap) {
  if (rows == 0 || n == 0) return cudaSuccess;
  CUtensorMap ma, mb;
  if (!tc::make_map(&ma, x, (uint64_t)K, (uint64_t)rows, (uint64_t)ldx, tc::BM) ||
      !tc::make_map(&mb, w, (uint64_t)kwrap, (uint64_t)n, (uint64_t)ldw, tc::BN))
    return cudaErrorInvalidValue;
  auto kern = tc::gemm_tc_kernel<Epi>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  const int64_t tiles = ceil_div(n, tc::BN) * ceil_div(rows, tc::BM);
  const int grid = (int)(tiles < tc::num_sms() ? tiles : tc::num_sms());
  LaunchScope scope_("gemm_tc", st);
  kern<<<grid, tc::THREADS, tc::SMEM_BYTES, st>>>(ma, mb, rows, K, n, epi, kwrap);
  return cudaGetLastError();
}

#define SDM_TC_INST(EPI)                                                                                         \
  template cudaError_t launch_gemm_tc<EPI>(const bf16_t*, int64_t, const bf16_t*, int64_t, int64_t, int, int, EPI, \
                                           cudaStream_t, int);
SDM_TC_INST(EpiF32)
SDM_TC_INST(EpiProj)
SDM_TC_INST(EpiStore<bf16_t>)
SDM_TC_INST(EpiF32R<bf16_t>)
SDM_TC_INST(EpiResid<bf16_t>)
SDM_TC_INST(EpiCE)
SDM_TC_INST(EpiArgmax)

// Read and clear the bounded-wait timeout flag (set by any kernel whose wait gave up).
cudaError_t read_and_clear_timeout(int* flag, cudaStream_t st) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(flag, g_tc_timeout, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return e;
  e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_tc_timeout, &zero, sizeof(int));
}

}  // namespace sdm
