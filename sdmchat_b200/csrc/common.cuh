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
