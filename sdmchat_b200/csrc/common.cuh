// Shared device helpers of the sm_100a SDM library.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include "../../include/sdm_b200.h"

namespace sdm {

typedef __nv_bfloat16 bf16_t;

// bfloat16 <-> float with round-to-nearest-even (the rounding torch's .to(torch.bfloat16) applies).
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(bf16_t x) { return __bfloat162float(x); }
template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ bf16_t from_f32<bf16_t>(float x) { return __float2bfloat16_rn(x); }
// Round a float to the precision of T (identity for float).
template <typename T> __device__ __forceinline__ float round_to(float x);
template <> __device__ __forceinline__ float round_to<float>(float x) { return x; }
template <> __device__ __forceinline__ float round_to<bf16_t>(float x) { return bf16_round(x); }

// x / d for several x over one d, from inv = __frcp_rn(d) (the correctly rounded reciprocal): the product x * inv
// corrected once by its exact residual, q + (x - q d) * inv with fused multiply-adds (Markstein's division step,
// which gives the correctly rounded quotient; tests/test_division_cpu.py checks it against IEEE division).  Three
// instructions per quotient instead of a full division each.
__device__ __forceinline__ float div_rn_by(float x, float d, float inv) {
  const float q = x * inv;
  return fmaf(fmaf(-q, d, x), inv, q);
}

// acc = a * b + acc on two float lanes at once (sm_100's paired FMA): each lane rounds exactly as fmaf does, so the
// results equal two scalar fmaf, at half the instructions.  The lanes are packed into 64-bit registers inside the
// asm (mov.b64 of a register pair), not by reinterpreting a float2 object's memory, which the compiler's alias
// analysis may order before the stores that fill it.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 acc) {
  float2 r;
  asm("{\n\t.reg .b64 pa, pb, pc, pd;\n\t"
      "mov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\tmov.b64 pc, {%6, %7};\n\t"
      "fma.rn.f32x2 pd, pa, pb, pc;\n\t"
      "mov.b64 {%0, %1}, pd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(acc.x), "f"(acc.y));
  return r;
}

// Correctly rounded 1/sqrt(v): sqrt then divide, both IEEE round-to-nearest, as the CPU reference computes
// torch.rsqrt (a square root and a division).
__device__ __forceinline__ float rsqrt_rn(float v) { return __fdiv_rn(1.0f, __fsqrt_rn(v)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Programmatic dependent launch.  Every kernel of the library is launched with launch_k and begins with
// pdl_enter(): wait until the kernel before it in the stream has completed with its writes visible (so every
// kernel has waited for its predecessor before it can complete, and the chain stays ordered), then allow the next
// kernel to start.  Small launches (decode: tens of rows, a fraction of one wave) get the programmatic attribute,
// so the next kernel's launch and block scheduling overlap this one's run; its blocks can be resident only once
// all of this kernel's blocks have started.  Large launches (prefill) keep plain stream order: their launch gaps
// are hidden by the second row stream, whose kernels early-resident waiting blocks would crowd out.  Both
// instructions are no-ops for a launch without the attribute.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
constexpr int64_t PDL_MAX_THREADS = 148 * 512;   // a quarter of the B200's resident threads
constexpr size_t PDL_MAX_SMEM = 48 * 1024;
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  const int64_t threads = (int64_t)grid.x * grid.y * grid.z * block.x * block.y * block.z;
  cfg.attrs = attr;
  cfg.numAttrs = (threads <= PDL_MAX_THREADS && smem <= PDL_MAX_SMEM) ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...);
}

// Every kernel launch sits inside a LaunchScope: it counts the launch (sdm_kernel_launch_count) and, while
// sdm_profile_begin/end is recording, brackets it with CUDA events on the launch stream, grouped by kernel name
// and the call-site tag of the innermost OpTag.
struct LaunchScope {
  LaunchScope(const char* kernel, cudaStream_t st);
  ~LaunchScope();
  int rec_;
  cudaStream_t st_;
};
struct OpTag {
  explicit OpTag(const char* tag);
  ~OpTag();
  const char* prev_;
};

}  // namespace sdm

// Host-side status helpers.
#define SDM_CHECK_LAUNCH()                                   \
  do {                                                       \
    cudaError_t e_ = cudaGetLastError();                     \
    if (e_ != cudaSuccess) return SDM_ERR_CUDA;              \
  } while (0)
#define SDM_REQUIRE(cond, code) \
  do {                          \
    if (!(cond)) return (code); \
  } while (0)
