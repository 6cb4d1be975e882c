// mbarrier and TMA helpers shared by the kernels that stage operands with the Tensor Memory Accelerator.
// Every copy here lands in the issuing CTA's own shared memory, and every wait is bounded.
#pragma once
#include <cuda.h>
#include "common.cuh"

namespace sdm {
namespace tma {

// Set by a bounded wait that gave up (one copy per .cu module; read back through that module's host function).
static __device__ int g_wait_timeout;
// How long a bounded wait keeps polling before it gives up, in ns of %globaltimer (one copy per .cu module; set
// through set_wait_limit, e.g. shortened by a test that makes a wait run out).
constexpr unsigned long long kDefaultWaitLimitNs = 4000000000ull;
static __device__ unsigned long long g_wait_limit_ns = kDefaultWaitLimitNs;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
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
// Wait for the phase with the given parity to complete; false (and the timeout flag set) once g_wait_limit_ns
// (about 4 s unless changed) has passed.
static __device__ __noinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  const uint64_t limit = *(volatile unsigned long long*)&g_wait_limit_ns;
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > limit) {
      atomicExch(&g_wait_timeout, 1);
      return false;
    }
  }
}

// Orders this thread's earlier generic-proxy accesses of shared memory before its later async-proxy (TMA) ones.
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Brings a tensor map (kernel parameter) into the TMA descriptor cache ahead of its first use.
__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled tensor load into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void load_2d(const CUtensorMap* map, uint64_t* bar, void* dst, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// Contiguous bulk load of `bytes` (a multiple of 16; both addresses 16-byte aligned) completing on `bar`.
__device__ __forceinline__ void load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Reads and clears this module's timeout flag (synchronises the stream).
static inline cudaError_t read_and_clear_wait_timeout(int* flag, cudaStream_t st) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(flag, g_wait_timeout, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) return e;
  e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(g_wait_timeout, &zero, sizeof(int));
}

// Sets this module's bounded-wait limit on the current device (0 restores the default); synchronous.
static inline cudaError_t set_wait_limit(unsigned long long ns) {
  const unsigned long long v = ns ? ns : kDefaultWaitLimitNs;
  return cudaMemcpyToSymbol(g_wait_limit_ns, &v, sizeof(v));
}

}  // namespace tma

// 2-D tensor map over a row-major (outer, inner) matrix of `dtype` elements with row stride ld_bytes; box
// (box_inner, box_outer) elements.  False when the driver entry point is unavailable or rejects the layout.
bool make_tensor_map_2d(CUtensorMap* m, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
                        uint64_t ld_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle);

}  // namespace sdm
