// bfloat16 GEMM on the sm_100a tensor cores: y = x @ w^T with a fused epilogue (tcgen05.mma, TMA, TMEM).
//
// Persistent kernel, one CTA per SM, CTA tile 128 x BN (BN = 256, or 128 when that keeps more SMs busy), K step 64
// (one 128-byte swizzle atom of bf16 per row).  Warp roles:
//   warp 0      TMA producer: one lane streams A (x rows) and B (w rows) tiles into a STAGES-deep ring with
//               cp.async.bulk.tensor, completing on the stage's `full` mbarrier.
//   warp 1      MMA issuer: allocates two BN-column TMEM accumulators; one lane issues 4 tcgen05.mma (K = 16 each)
//               per stage from shared-memory descriptors, releases the stage with tcgen05.commit on `empty` and,
//               after a tile's last stage, commits that accumulator's `acc_full` barrier.
//   warps 2-9   epilogue: warp w reads TMEM lanes 32*(w%4)..+31 (accumulator rows) and half (w-2)/4 of the tile's
//               columns, 32 columns per tcgen05.ld, then hands the accumulator back (`acc_empty`), so tile i's
//               epilogue runs while tile i+1's MMAs fill the other accumulator.
// Element-wise epilogues fetch their global inputs (biases, the residual input) for the whole tile before waiting
// for the accumulator, then pass each 32 x 32 block through a padded shared-memory transpose so every lane stores
// four consecutive columns (16-byte stores; eight lanes cover a 128-byte row segment).  Row-owned epilogues
// (kRowMode: the tied-head loss / argmax) reduce each thread's row of its 128 columns in registers and write one
// partial per (row, 128-column block).
// Every mbarrier wait is bounded (about 4 s of %globaltimer); a wait that gives up sets the module's timeout flag, every role
// falls through to the common exit, and the TMEM columns are released.  No load here reads another GPU's memory
// and none is issued to more than one CTA.
#include <cuda.h>
#include "kernels.cuh"
#include "tma.cuh"

namespace sdm {

namespace tc {

constexpr int BM = 128, BK = 64, EPI_WARPS = 8, THREADS = 64 + 32 * EPI_WARPS;
constexpr int STG_LD = 32;  // row (floats) of an epilogue warp's 32 x 32 transpose; float4 chunk j of row r sits
                            // at chunk j ^ (r & 7), so row writes and column reads are both conflict-free
constexpr uint32_t A_BYTES = BM * BK * 2;

// Ring depth: 4 stages (BN 256) / 6 (BN 128) -- the K = 1,536 residual GEMMs gain from the deeper ring -- except for
// the float32-output projection, measured faster with 3 / 5 (its epilogue, not operand latency, sets its pace).
template <typename Epi>
struct RingStages {
  static constexpr int deep = 1;
};
template <>
struct RingStages<EpiProj> {
  static constexpr int deep = 0;
};
template <int BN, int DEEP = 1>
struct Cfg {
  static constexpr int STAGES = (BN >= 256 ? 3 : 5) + DEEP;
  static constexpr uint32_t B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr size_t RING_BYTES = (size_t)STAGES * STAGE_BYTES;
  static constexpr size_t SMEM_BYTES = RING_BYTES + (size_t)EPI_WARPS * 32 * STG_LD * 4 + 1024;
  static constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulators (a power of two: 256 or 512)
  static constexpr int NCH = BN / 64;            // 32-column chunks per epilogue warp
  // Instruction descriptor of tcgen05.mma kind::f16: D float32, A and B bfloat16, both K-major, M = 128, N = BN.
  static constexpr uint32_t IDESC =
      (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
};

using namespace sdm::tma;

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: rows of 128 B, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;             // leading byte offset (unused by swizzled K-major layouts)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;             // descriptor version of sm_100
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
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

template <typename Epi, int BN>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int64_t rows,
                   int K, int n, Epi epi, int kwrap) {
  pdl_enter();
  using C = Cfg<BN, RingStages<Epi>::deep>;
  extern __shared__ __align__(1024) unsigned char dsmem[];
  __shared__ __align__(8) uint64_t full_bar[C::STAGES];
  __shared__ __align__(8) uint64_t empty_bar[C::STAGES];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ uint32_t tmem_slot;

  unsigned char* ring = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~(uintptr_t)1023);
  float* stage_all = reinterpret_cast<float*>(ring + C::RING_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt_count = (K + BK - 1) / BK;
  const int tiles_n = (n + BN - 1) / BN;
  const int64_t tiles = (int64_t)tiles_n * ((rows + BM - 1) / BM);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], EPI_WARPS);  // one arrival per epilogue warp
    }
    mbar_init_fence();
    prefetch_map(&tmA);
    prefetch_map(&tmB);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(C::TMEM_COLS)
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
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1u;
          if (!mbar_wait(&empty_bar[s], ph ^ 1u)) {
            ok = false;
            break;
          }
          unsigned char* a_dst = ring + s * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full_bar[s], C::STAGE_BYTES);
          load_2d(&tmA, &full_bar[s], a_dst, kt * BK, m0);
          load_2d(&tmB, &full_bar[s], a_dst + A_BYTES, (kt * BK) % kwrap, n0);
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
        // a last column tile narrower than BN multiplies only its columns (rounded up to 16; the box's rows past n
        // are zero-filled): N is field 17-22 of the instruction descriptor
        const int nrem = n - (int)(t % tiles_n) * BN;
        const int nt = nrem >= BN ? BN : ((nrem + 15) & ~15);
        const uint32_t idesc = (C::IDESC & ~(0x3Fu << 17)) | ((uint32_t)(nt >> 3) << 17);
        for (int kt = 0; kt < kt_count; ++kt, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1u;
          if (!mbar_wait(&full_bar[s], ph)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a_base = smem_u32(ring + s * C::STAGE_BYTES);
          const uint32_t b_base = a_base + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_bf16(dt, sw128_desc(a_base + kk * 32), sw128_desc(b_base + kk * 32), idesc, (kt | kk) != 0);
          umma_commit(&empty_bar[s]);
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
    }
  } else {
    // epilogue warps 2..9: TMEM lane quarter q = warp % 4, column half of the tile `half`
    const int ew = warp - 2, q = warp & 3, half = ew >> 2;
    float* stg = stage_all + ew * 32 * STG_LD;
    const int rsub = lane >> 3, c4 = lane & 7;
    uint32_t tl = 0;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++tl) {
      const uint32_t buf = tl & 1u, use = tl >> 1;
      const int tn = (int)(t % tiles_n);
      const int64_t m0 = (t / tiles_n) * BM;
      const int64_t row0 = m0 + q * 32;
      const int cb = tn * BN + half * (BN / 2);  // first column of this warp's half
      const uint32_t taddr = tmem + buf * BN + ((uint32_t)(q * 32) << 16) + (uint32_t)(half * (BN / 2));
      if constexpr (Epi::kRowMode) {
        if (!mbar_wait(&acc_full[buf], use & 1u)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        typename Epi::RowState rs;
        epi.row_begin(rs, row0 + lane, rows, cb);
#pragma unroll 1
        for (int ch = 0; ch < C::NCH; ++ch) {
          uint32_t r[32];
          tmem_ld32(taddr + (uint32_t)(ch * 32), r);
          epi.row_chunk(rs, cb + ch * 32, n, r);
        }
        if (cb < n) epi.row_end(rs, row0 + lane, rows, cb / (BN / 2), (n + BN / 2 - 1) / (BN / 2));
      } else {
        // the tile's epilogue inputs first: they arrive while the MMAs run
        typename Epi::Pre pre[C::NCH];
        const int64_t rl0 = row0 + rsub;
#pragma unroll
        for (int ch = 0; ch < C::NCH; ++ch) epi.prefetch(pre[ch], rl0, rows, cb + ch * 32 + 4 * c4, n);
        if (!mbar_wait(&acc_full[buf], use & 1u)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
        for (int ch = 0; ch < C::NCH; ++ch) {
          uint32_t r[32];
          tmem_ld32(taddr + (uint32_t)(ch * 32), r);
          float4* srow = reinterpret_cast<float4*>(stg + lane * STG_LD);  // this thread's row
#pragma unroll
          for (int j = 0; j < 8; ++j)
            srow[j ^ (lane & 7)] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                               __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
          __syncwarp();
          const int col = cb + ch * 32 + 4 * c4;
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int rr = 4 * it + rsub;
            const float4 v = *reinterpret_cast<const float4*>(stg + rr * STG_LD + 4 * (c4 ^ (rr & 7)));
            if (row0 + rr < rows && col < n) epi.store4(pre[ch], it, row0 + rr, col, v, n);
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
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS) : "memory");
  }
}

// ------------------------------------------------------------------------------------------------ CTA pairs
// The same GEMM on pairs of CTAs (a cluster of two, tcgen05 cta_group::2): the pair owns a 256 x 256 tile, each CTA
// stages its 128 rows of A and its 128 rows of B (one half of the tile's columns) per K step, and one thread of the
// even CTA issues 256 x N x 16 MMAs that read both CTAs' shared memory and leave each CTA's 128 rows of the
// accumulator in its own TMEM.  Per CTA and K step 32 KB of operands feed 128 x 256 outputs (48 KB in the
// single-CTA tile), so the L2 -> SM operand traffic per flop falls by a third.  Loads are plain TMA tile loads,
// each into its own CTA; they complete on the even CTA's `full` barrier, whose expected bytes cover both halves.
// The MMA thread commits each consumed stage to the even CTA's `empty` barrier, whose producer passes the release on
// to the odd CTA's, and each finished accumulator to both CTAs' `acc_full`; every epilogue warp of both
// CTAs arrives on the even CTA's `acc_empty`.  All waits are the bounded mbarrier waits; the two cluster barriers
// (after set-up, before TMEM release) are reached on every path.
// SPLIT (K = 2 x kwrap, x = [hi | lo] against one w): a stage holds the hi and the lo A tiles of one K block and
// the one B tile both multiply, so each weight tile crosses L2 -> SMEM once instead of twice (the kernel is bound by
// that operand traffic: its MMA thread waits on `full` for about 40 % of its time, on the accumulators for about 3 %).
constexpr int PAIR_N = 256;
template <int DEEP, bool SPLIT = false>
struct Cfg2 {
  static constexpr int STAGES = SPLIT ? 4 : 5 + DEEP;
  static constexpr uint32_t B_BYTES = (PAIR_N / 2) * BK * 2, STAGE_BYTES = (SPLIT ? 2 : 1) * A_BYTES + B_BYTES;
  static constexpr size_t RING_BYTES = (size_t)STAGES * STAGE_BYTES;
  static constexpr size_t SMEM_BYTES = RING_BYTES + (size_t)EPI_WARPS * 32 * STG_LD * 4 + 1024;
  static constexpr uint32_t TMEM_COLS = 2 * PAIR_N;
  static constexpr int NCH = PAIR_N / 64;
  // kind::f16: D float32, A and B bfloat16, both K-major, M = 256 (the pair), N = 256
  static constexpr uint32_t IDESC =
      (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(PAIR_N >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Shared::cluster address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 2-D tile load into this CTA's shared memory only, completing on an mbarrier of either CTA of the pair.
__device__ __forceinline__ void load_2d_pair(const CUtensorMap* map, uint32_t mbar_cluster, void* dst, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar_cluster)
      : "memory");
}
__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}
// Arrives on `bar` in this (the even) CTA when the issued MMAs have completed.
__device__ __forceinline__ void umma_commit_own(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(peer_addr(bar, 0))
               : "memory");
}
// Arrives once on `bar` (the same offset) in both CTAs of the pair when the issued MMAs have completed: one
// commit per CTA's barrier (each tracks every MMA this thread issued before it).
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(peer_addr(bar, 0))
               : "memory");
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(peer_addr(bar, 1))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

template <typename Epi, bool SPLIT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int64_t rows,
                    int K, int n, Epi epi, int kwrap) {
  pdl_enter();
  using C = Cfg2<RingStages<Epi>::deep, SPLIT>;
  constexpr uint32_t B_OFF = (SPLIT ? 2 : 1) * A_BYTES;  // the B tile's offset in a stage
  extern __shared__ __align__(1024) unsigned char dsmem[];
  __shared__ __align__(8) uint64_t full_bar[C::STAGES];
  __shared__ __align__(8) uint64_t empty_bar[C::STAGES];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ uint32_t tmem_slot;

  unsigned char* ring = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~(uintptr_t)1023);
  float* stage_all = reinterpret_cast<float*>(ring + C::RING_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int64_t pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int kt_count = ((SPLIT ? kwrap : K) + BK - 1) / BK;
  const int tiles_n = (n + PAIR_N - 1) / PAIR_N;
  const int64_t tiles = (int64_t)tiles_n * ((rows + 2 * BM - 1) / (2 * BM));

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);   // the even CTA's producer (expect_tx of both halves)
      mbar_init(&empty_bar[s], 1);  // the pair's MMA commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 2 * EPI_WARPS);  // every epilogue warp of both CTAs
    }
    mbar_init_fence();
    prefetch_map(&tmA);
    prefetch_map(&tmB);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(C::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated before any copy or MMA
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int64_t t = pair; t < tiles && ok; t += npairs) {
        const int tn = (int)(t % tiles_n);
        const int m0 = (int)(t / tiles_n) * 2 * BM + (int)rank * BM;
        const int nrem = n - tn * PAIR_N;
        const int nt = nrem >= PAIR_N ? PAIR_N : ((nrem + 31) & ~31);
        const int nb = tn * PAIR_N + (int)rank * (nt >> 1);
        for (int kt = 0; kt < kt_count; ++kt, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1u;
          if (!mbar_wait(&empty_bar[s], ph ^ 1u)) {
            ok = false;
            break;
          }
          // the MMA thread commits a consumed stage to the even CTA's `empty` only; its producer passes each
          // release on to the odd CTA's `empty`, one arrival per reuse of the stage
          if (leader && it >= (uint32_t)C::STAGES) mbar_arrive_remote(peer_addr(&empty_bar[s], 1));
          unsigned char* a_dst = ring + s * C::STAGE_BYTES;
          if (leader) mbar_arrive_expect_tx(&full_bar[s], 2 * C::STAGE_BYTES);
          const uint32_t fb = peer_addr(&full_bar[s], 0);
          load_2d_pair(&tmA, fb, a_dst, kt * BK, m0);
          if constexpr (SPLIT) load_2d_pair(&tmA, fb, a_dst + A_BYTES, kt * BK + kwrap, m0);
          load_2d_pair(&tmB, fb, a_dst + B_OFF, (kt * BK) % kwrap, nb);
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      uint32_t it = 0, tl = 0;
      bool ok = true;
      for (int64_t t = pair; t < tiles && ok; t += npairs, ++tl) {
        const uint32_t buf = tl & 1u, use = tl >> 1;
        if (!mbar_wait(&acc_empty[buf], (use & 1u) ^ 1u)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t dt = tmem + buf * PAIR_N;
        const int nrem = n - (int)(t % tiles_n) * PAIR_N;
        const int nt = nrem >= PAIR_N ? PAIR_N : ((nrem + 31) & ~31);
        const uint32_t idesc = (C::IDESC & ~(0x3Fu << 17)) | ((uint32_t)(nt >> 3) << 17);
        for (int kt = 0; kt < kt_count; ++kt, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1u;
          if (!mbar_wait(&full_bar[s], ph)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a_base = smem_u32(ring + s * C::STAGE_BYTES);
          const uint32_t b_base = a_base + B_OFF;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_bf16_pair(dt, sw128_desc(a_base + kk * 32), sw128_desc(b_base + kk * 32), idesc, (kt | kk) != 0);
          if constexpr (SPLIT) {  // the lo half of the same K block against the same weights
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              umma_bf16_pair(dt, sw128_desc(a_base + A_BYTES + kk * 32), sw128_desc(b_base + kk * 32), idesc, 1u);
          }
          umma_commit_own(&empty_bar[s]);
        }
        if (ok) umma_commit_pair(&acc_full[buf]);
      }
    }
  } else {
    const int ew = warp - 2, q = warp & 3, half = ew >> 2;
    float* stg = stage_all + ew * 32 * STG_LD;
    const int rsub = lane >> 3, c4 = lane & 7;
    const uint32_t release = peer_addr(&acc_empty[0], 0);  // acc_empty[buf] of the even CTA: + 8 * buf
    uint32_t tl = 0;
    for (int64_t t = pair; t < tiles; t += npairs, ++tl) {
      const uint32_t buf = tl & 1u, use = tl >> 1;
      const int tn = (int)(t % tiles_n);
      const int64_t m0 = (t / tiles_n) * 2 * BM + (int64_t)rank * BM;
      const int64_t row0 = m0 + q * 32;
      const int cb = tn * PAIR_N + half * (PAIR_N / 2);
      const uint32_t taddr = tmem + buf * PAIR_N + ((uint32_t)(q * 32) << 16) + (uint32_t)(half * (PAIR_N / 2));
      if constexpr (Epi::kRowMode) {
        if (!mbar_wait(&acc_full[buf], use & 1u)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        typename Epi::RowState rs;
        epi.row_begin(rs, row0 + lane, rows, cb);
#pragma unroll 1
        for (int ch = 0; ch < C::NCH; ++ch) {
          uint32_t r[32];
          tmem_ld32(taddr + (uint32_t)(ch * 32), r);
          epi.row_chunk(rs, cb + ch * 32, n, r);
        }
        if (cb < n) epi.row_end(rs, row0 + lane, rows, cb / (PAIR_N / 2), (n + PAIR_N / 2 - 1) / (PAIR_N / 2));
      } else {
        typename Epi::Pre pre[C::NCH];
        const int64_t rl0 = row0 + rsub;
#pragma unroll
        for (int ch = 0; ch < C::NCH; ++ch) epi.prefetch(pre[ch], rl0, rows, cb + ch * 32 + 4 * c4, n);
        if (!mbar_wait(&acc_full[buf], use & 1u)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
        for (int ch = 0; ch < C::NCH; ++ch) {
          uint32_t r[32];
          tmem_ld32(taddr + (uint32_t)(ch * 32), r);
          float4* srow = reinterpret_cast<float4*>(stg + lane * STG_LD);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            srow[j ^ (lane & 7)] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                               __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
          __syncwarp();
          const int col = cb + ch * 32 + 4 * c4;
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int rr = 4 * it + rsub;
            const float4 v = *reinterpret_cast<const float4*>(stg + rr * STG_LD + 4 * (c4 ^ (rr & 7)));
            if (row0 + rr < rows && col < n) epi.store4(pre[ch], it, row0 + rr, col, v, n);
          }
          __syncwarp();
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(release + 8u * buf);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  cluster_sync_all();  // no MMA of the pair still reads this CTA's shared memory or writes its TMEM
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS) : "memory");
  }
}

// 2-D bf16 tensor map over a row-major (outer, inner) matrix with row stride ld elements; box (64, box_outer),
// 128-byte swizzle (the UMMA K-major operand layout).
static bool make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_outer) {
  return make_tensor_map_2d(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, inner, outer, ld * 2, (uint32_t)BK, box_outer,
                            CU_TENSOR_MAP_SWIZZLE_128B);
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

bool make_tensor_map_2d(CUtensorMap* m, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
                        uint64_t ld_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  return fn(m, dtype, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tc_gemm_supported(const void* x, int64_t ldx, const void* w, int64_t ldw, int K, int kwrap) {
  const uintptr_t ax = reinterpret_cast<uintptr_t>(x), aw = reinterpret_cast<uintptr_t>(w);
  const bool wrap_ok = kwrap == K || (kwrap % tc::BK) == 0;  // a wrapped B restarts on a K-step boundary
  return K >= 16 && (K % 8) == 0 && wrap_ok && (ax % 16) == 0 && (aw % 16) == 0 && (ldx % 8) == 0 &&
         (ldw % 8) == 0 && encode_fn() != nullptr;
}

template <typename Epi, int BN>
static cudaError_t launch_tc_bn(const bf16_t* x, int64_t ldx, const bf16_t* w, int64_t ldw, int64_t rows, int K,
                                int n, Epi epi, cudaStream_t st, int kwrap) {
  using C = tc::Cfg<BN, tc::RingStages<Epi>::deep>;
  CUtensorMap ma, mb;
  if (!tc::make_map(&ma, x, (uint64_t)K, (uint64_t)rows, (uint64_t)ldx, tc::BM) ||
      !tc::make_map(&mb, w, (uint64_t)kwrap, (uint64_t)n, (uint64_t)ldw, BN))
    return cudaErrorInvalidValue;
  auto kern = tc::gemm_tc_kernel<Epi, BN>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  // as few CTAs as finish the tiles in the same number of rounds: the SMs left over stay free for kernels of other
  // streams (rows split over streams run side by side)
  const int64_t tiles = ceil_div(n, BN) * ceil_div(rows, tc::BM);
  const int64_t rounds = ceil_div(tiles, (int64_t)tc::num_sms());
  const int grid = (int)ceil_div(tiles, rounds);
  LaunchScope scope_("gemm_tc", st);
  return launch_k(kern, dim3(grid), dim3(tc::THREADS), C::SMEM_BYTES, st, ma, mb, rows, K, n, epi, kwrap);
}

// CTA-pair launch: clusters of two, as many pairs as fit at once (the persistent loop covers the rest).
template <typename Epi, bool SPLIT>
static cudaError_t launch_tc_pair_k(const bf16_t* x, int64_t ldx, const bf16_t* w, int64_t ldw, int64_t rows, int K,
                                    int n, Epi epi, cudaStream_t st, int kwrap) {
  using C = tc::Cfg2<tc::RingStages<Epi>::deep, SPLIT>;
  CUtensorMap ma, mb;
  if (!tc::make_map(&ma, x, (uint64_t)K, (uint64_t)rows, (uint64_t)ldx, tc::BM) ||
      !tc::make_map(&mb, w, (uint64_t)kwrap, (uint64_t)n, (uint64_t)ldw, tc::PAIR_N / 2))
    return cudaErrorInvalidValue;
  auto kern = tc::gemm_tc2_kernel<Epi, SPLIT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM_BYTES);
  if (e != cudaSuccess) return e;
  static int max_pairs[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int pairs_cap = tc::num_sms() / 2;
  if (dev >= 0 && dev < 64) {
    if (!max_pairs[dev]) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * pairs_cap);
      cfg.blockDim = dim3(tc::THREADS);
      cfg.dynamicSmemBytes = C::SMEM_BYTES;
      int nc = 0;
      max_pairs[dev] = (cudaOccupancyMaxActiveClusters(&nc, kern, &cfg) == cudaSuccess && nc > 0) ? nc : pairs_cap;
      cudaGetLastError();
    }
    pairs_cap = max_pairs[dev] < pairs_cap ? max_pairs[dev] : pairs_cap;
  }
  const int64_t tiles = ceil_div(n, tc::PAIR_N) * ceil_div(rows, 2 * tc::BM);
  const int pairs = (int)ceil_div(tiles, ceil_div(tiles, (int64_t)pairs_cap));  // same rounds, fewest pairs
  LaunchScope scope_("gemm_tc", st);
  return launch_k(kern, dim3(2 * pairs), dim3(tc::THREADS), C::SMEM_BYTES, st, ma, mb, rows, K, n, epi, kwrap);
}
// A [hi | lo] input against one weight (K = 2 x kwrap) takes the split stages.
template <typename Epi>
static cudaError_t launch_tc_pair(const bf16_t* x, int64_t ldx, const bf16_t* w, int64_t ldw, int64_t rows, int K,
                                  int n, Epi epi, cudaStream_t st, int kwrap) {
  if (K == 2 * kwrap && kwrap % tc::BK == 0)
    return launch_tc_pair_k<Epi, true>(x, ldx, w, ldw, rows, K, n, epi, st, kwrap);
  return launch_tc_pair_k<Epi, false>(x, ldx, w, ldw, rows, K, n, epi, st, kwrap);
}

// Column tile: 256 wide moves a third fewer operand bytes per flop; 128 wide when it finishes in fewer rounds of
// persistent tiles (small problems).  Row-owned epilogues always take 256 (two 128-column partials per tile).  A
// 256-wide tile over at least 256 rows runs on CTA pairs (256 x 256 per pair).
template <typename Epi>
cudaError_t launch_gemm_tc(const bf16_t* x, int64_t ldx, const bf16_t* w, int64_t ldw, int64_t rows, int K, int n,
                           Epi epi, cudaStream_t st, int kwrap) {
  if (rows == 0 || n == 0) return cudaSuccess;
  if constexpr (Epi::kRowMode) {
    if (rows >= 2 * tc::BM) return launch_tc_pair<Epi>(x, ldx, w, ldw, rows, K, n, epi, st, kwrap);
    return launch_tc_bn<Epi, 256>(x, ldx, w, ldw, rows, K, n, epi, st, kwrap);
  } else {
    const int64_t sms = tc::num_sms(), mt = ceil_div(rows, tc::BM);
    const int64_t rounds256 = ceil_div(mt * ceil_div(n, 256), sms), rounds128 = ceil_div(mt * ceil_div(n, 128), sms);
    if (rounds256 * 256 * 3 <= rounds128 * 128 * 4) {  // a 256-wide round costs about 1.5x a 128-wide one
      if (rows >= 2 * tc::BM) return launch_tc_pair<Epi>(x, ldx, w, ldw, rows, K, n, epi, st, kwrap);
      return launch_tc_bn<Epi, 256>(x, ldx, w, ldw, rows, K, n, epi, st, kwrap);
    }
    return launch_tc_bn<Epi, 128>(x, ldx, w, ldw, rows, K, n, epi, st, kwrap);
  }
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
SDM_TC_INST(EpiSwiGLU)

// Read and clear the bounded-wait timeout flag of the GEMM module.
cudaError_t read_and_clear_timeout(int* flag, cudaStream_t st) { return tma::read_and_clear_wait_timeout(flag, st); }
cudaError_t set_gemm_wait_limit(unsigned long long ns) { return tma::set_wait_limit(ns); }

// One thread waits, through the GEMM's bounded mbarrier wait, on a barrier that nothing arrives on and that no
// copy completes: the wait gives up after the module's limit, sets the timeout flag and the kernel returns.
__global__ void wait_probe_kernel(int* done) {
  pdl_enter();
  __shared__ __align__(8) uint64_t bar;
  tma::mbar_init(&bar, 1);
  tma::mbar_init_fence();
  const bool ok = tma::mbar_wait(&bar, 0u);
  *done = ok ? 1 : 2;
}
cudaError_t launch_wait_probe(int* done, cudaStream_t st) {
  LaunchScope scope_("wait_probe", st);
  return launch_k(wait_probe_kernel, dim3(1), dim3(1), 0, st, done);
}

}  // namespace sdm
