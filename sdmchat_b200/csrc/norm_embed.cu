// RMSNorm, token-table lookup, SwiGLU activation, RunTimeSdm finish and TrainedSdm value gather.
#include "pk_common.cuh"

namespace sdm {

// RMSNorm.forward (track4_sdmllm_models.py:69-71): y = (x * rsqrt(mean x^2 + eps)).to(T) * w, one warp per row.
// In bfloat16 the normalised value is rounded before the weight product, whose result is rounded again.
template <typename T>
__global__ void rmsnorm_kernel(const T* __restrict__ x, const T* __restrict__ w, int64_t rows, int d, float eps,
                               T* __restrict__ y) {
  pdl_enter();
  int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + row * d;
  float ss = 0.f;
  for (int c = lane; c < d; c += 32) {
    float v = to_f32(xr[c]);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  float r = rsqrt_rn(__fdiv_rn(ss, (float)d) + eps);
  T* yr = y + row * d;
  for (int c = lane; c < d; c += 32) {
    float v = round_to<T>(to_f32(xr[c]) * r);
    yr[c] = from_f32<T>(v * to_f32(w[c]));
  }
}

// The same RMSNorm with the row held in registers: each lane loads NCH 16-byte chunks (chunk q of lane l covers
// columns (l + 32 q) * E .. +E-1, E = 16 / sizeof(T)), so x is read once with coalesced 16-byte accesses.
template <typename T, int NCH>
__global__ void rmsnorm_vec_kernel(const T* __restrict__ x, const T* __restrict__ w, int64_t rows, float eps,
                                   T* __restrict__ y) {
  pdl_enter();
  constexpr int E = 16 / sizeof(T), D = NCH * 32 * E;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * D);
  uint4 raw[NCH];
#pragma unroll
  for (int q = 0; q < NCH; ++q) raw[q] = xr[lane + 32 * q];
  float ss = 0.f;
#pragma unroll
  for (int q = 0; q < NCH; ++q) {
    const T* v = reinterpret_cast<const T*>(&raw[q]);
#pragma unroll
    for (int e = 0; e < E; ++e) ss = fmaf(to_f32(v[e]), to_f32(v[e]), ss);
  }
  ss = warp_sum(ss);
  const float r = rsqrt_rn(__fdiv_rn(ss, (float)D) + eps);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* yr = reinterpret_cast<uint4*>(y + row * D);
#pragma unroll
  for (int q = 0; q < NCH; ++q) {
    const uint4 wv = wr[lane + 32 * q];
    const T* v = reinterpret_cast<const T*>(&raw[q]);
    const T* wt = reinterpret_cast<const T*>(&wv);
    uint4 out;
    T* o = reinterpret_cast<T*>(&out);
#pragma unroll
    for (int e = 0; e < E; ++e) o[e] = from_f32<T>(round_to<T>(to_f32(v[e]) * r) * to_f32(wt[e]));
    yr[lane + 32 * q] = out;
  }
}

template <typename T>
__global__ void embed_kernel(const int32_t* __restrict__ ids, const T* __restrict__ emb, int64_t N, int d, int V,
                             T* __restrict__ out, int* bad) {
  pdl_enter();
  int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (row >= N) return;
  int id = ids[row];
  bool ok = id >= 0 && id < V;
  if (!ok && lane == 0 && bad) atomicExch(bad, 1);
  for (int c = lane; c < d; c += 32) out[row * d + c] = ok ? emb[(int64_t)id * d + c] : from_f32<T>(0.f);
}

// SwiGLU activation (track4_sdmllm_models.py:96-97): p = silu(g) * u with the bf16 roundings of a bf16 module.
template <typename T>
__global__ void swiglu_act_kernel(const T* __restrict__ gu, int64_t rows, int f, T* __restrict__ p) {
  // gu (rows, 2f) in the packed layout of swiglu_pack_rows: output column j reads gate column 32*(j/16) + j%16 and
  // up column 16 further
  pdl_enter();
  const int64_t n = rows * f;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    const int64_t r = i / f;
    const int j = (int)(i - r * f);
    const T* row = gu + r * 2 * f + 32 * (j >> 4) + (j & 15);
    const float gv = to_f32(row[0]);
    const float s = round_to<T>(gv / (1.f + expf(-gv)));
    p[i] = from_f32<T>(s * to_f32(row[16]));
  }
}

// Store v at row n, column c of a row of width d: plain, or as bfloat16 hi (column c) + lo (column d + c).
template <typename T>
__device__ __forceinline__ void store_split(T* r, int64_t n, int64_t d, int64_t c, float v, int split) {
  if (split) {
    const float hi = round_to<T>(v);
    r[n * 2 * d + c] = from_f32<T>(hi);
    r[n * 2 * d + d + c] = from_f32<T>(v - hi);
  } else {
    r[n * d + c] = from_f32<T>(v);
  }
}

// Four consecutive columns c..c+3 (c a multiple of 4) of store_split: 8-byte bf16 stores (16-byte float32) when the
// destination is aligned.
template <typename T>
__device__ __forceinline__ void store_split4(T* r, int64_t n, int64_t d, int64_t c, float4 v, int split) {
  if (split) {
    const float4 hi = make_float4(round_to<T>(v.x), round_to<T>(v.y), round_to<T>(v.z), round_to<T>(v.w));
    store4_to(r + n * 2 * d + c, hi, 4);
    store4_to(r + n * 2 * d + d + c, make_float4(v.x - hi.x, v.y - hi.y, v.z - hi.z, v.w - hi.w), 4);
  } else {
    store4_to(r + n * d + c, v, 4);
  }
}

// RunTimeSdm.finish up to wo (track4_onesdm_models.py:243-246): mean (or sum) read, per-head RMS out-norm with
// onorm_w.  num (N, h, dh), den (N, h) float32 -> r (N, h*dh) in T.  One warp per (token, head).
template <typename T>
__global__ void rt_finish_kernel(const float* __restrict__ num, const float* __restrict__ den, int64_t N, int h,
                                 int dh, int read_sum, float read_eps, int out_norm, float out_norm_eps,
                                 const float* __restrict__ onorm_w, T* __restrict__ r, int split) {
  pdl_enter();
  int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (item >= N * h) return;
  int hh = (int)(item % h);
  const float* nr = num + item * dh;
  float dv = read_sum ? 0.f : den[item] + read_eps;
  float vals[8];
  float ss = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    int c = lane + 32 * q;
    float v = 0.f;
    if (c < dh) {
      v = read_sum ? nr[c] : __fdiv_rn(nr[c], dv);
      ss = fmaf(v, v, ss);
    }
    vals[q] = v;
  }
  float rs = 1.f;
  if (out_norm) rs = rsqrt_rn(__fdiv_rn(warp_sum(ss), (float)dh) + out_norm_eps);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    int c = lane + 32 * q;
    if (c < dh) {
      float v = vals[q];
      if (out_norm) v = (v * rs) * onorm_w[hh * dh + c];
      store_split<T>(r, item / h, (int64_t)h * dh, hh * dh + c, v, split);
    }
  }
}

// The same finish for dh = 32 * STEPS: eight lanes per (token, head) row, each lane 4 consecutive columns per
// 32-column step (16-byte loads), the row's sum of squares reduced over the eight lanes.  A lane group takes
// FIN_ROWS consecutive rows (4 for large launches, 1 for decode-sized ones) and issues all their loads before the
// first use, so the loads overlap.
template <typename T, int STEPS, int FIN_ROWS>
__global__ void __launch_bounds__(256) rt_finish_vec_kernel(const float* __restrict__ num, const float* __restrict__ den,
                                                            int64_t N, int h, int read_sum, float read_eps,
                                                            int out_norm, float out_norm_eps,
                                                            const float* __restrict__ onorm_w, T* __restrict__ r,
                                                            int split) {
  pdl_enter();
  constexpr int dh = 32 * STEPS;
  const int64_t item0 = (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3) * FIN_ROWS;
  const int g = threadIdx.x & 7;
  const int64_t items = N * h;
  float4 vals[FIN_ROWS][STEPS];
  float dv[FIN_ROWS];
#pragma unroll
  for (int i = 0; i < FIN_ROWS; ++i) {
    const int64_t it = item0 + i < items ? item0 + i : items - 1;
    const float4* nr = reinterpret_cast<const float4*>(num + it * dh);
#pragma unroll
    for (int q = 0; q < STEPS; ++q) vals[i][q] = nr[g * STEPS + q];  // lane g: columns g*dh/8 .. +dh/8-1
    dv[i] = read_sum ? 0.f : den[it] + read_eps;
  }
  float inv[FIN_ROWS];
#pragma unroll
  for (int i = 0; i < FIN_ROWS; ++i) inv[i] = read_sum ? 1.f : __frcp_rn(dv[i]);
#pragma unroll
  for (int i = 0; i < FIN_ROWS; ++i) {
    float ss = 0.f;
#pragma unroll
    for (int q = 0; q < STEPS; ++q) {
      float4 v = vals[i][q];
      if (!read_sum) {
        v.x = div_rn_by(v.x, dv[i], inv[i]);
        v.y = div_rn_by(v.y, dv[i], inv[i]);
        v.z = div_rn_by(v.z, dv[i], inv[i]);
        v.w = div_rn_by(v.w, dv[i], inv[i]);
      }
      ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
      vals[i][q] = v;
    }
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    ss += __shfl_xor_sync(0xffffffffu, ss, 4);
    const int64_t item = item0 + i;
    if (item >= items) continue;
    const int hh = (int)(item % h);
    const float rs = out_norm ? rsqrt_rn(__fdiv_rn(ss, (float)dh) + out_norm_eps) : 1.f;
    const int64_t n = item / h;
    float4 o[STEPS];
#pragma unroll
    for (int q = 0; q < STEPS; ++q) {
      const int c = (g * STEPS + q) * 4;
      o[q] = vals[i][q];
      if (out_norm) {
        const float4 wv = *reinterpret_cast<const float4*>(onorm_w + hh * dh + c);
        o[q] = make_float4((o[q].x * rs) * wv.x, (o[q].y * rs) * wv.y, (o[q].z * rs) * wv.z, (o[q].w * rs) * wv.w);
      }
    }
    if constexpr (sizeof(T) == 2 && STEPS % 2 == 0) {
      if (split) {  // eight consecutive columns per 16-byte store, hi and lo rows (the launcher checks alignment)
        const int64_t d = (int64_t)h * dh;
#pragma unroll
        for (int q = 0; q < STEPS; q += 2) {
          const float4 h0 = make_float4(round_to<T>(o[q].x), round_to<T>(o[q].y), round_to<T>(o[q].z), round_to<T>(o[q].w));
          const float4 h1 = make_float4(round_to<T>(o[q + 1].x), round_to<T>(o[q + 1].y), round_to<T>(o[q + 1].z),
                                        round_to<T>(o[q + 1].w));
          const float4 l0 = make_float4(o[q].x - h0.x, o[q].y - h0.y, o[q].z - h0.z, o[q].w - h0.w);
          const float4 l1 = make_float4(o[q + 1].x - h1.x, o[q + 1].y - h1.y, o[q + 1].z - h1.z, o[q + 1].w - h1.w);
          const uint2 ph0 = pack_bf16x4(h0), ph1 = pack_bf16x4(h1), pl0 = pack_bf16x4(l0), pl1 = pack_bf16x4(l1);
          T* dst = r + n * 2 * d + (int64_t)hh * dh + (g * STEPS + q) * 4;
          *reinterpret_cast<uint4*>(dst) = make_uint4(ph0.x, ph0.y, ph1.x, ph1.y);
          *reinterpret_cast<uint4*>(dst + d) = make_uint4(pl0.x, pl0.y, pl1.x, pl1.y);
        }
        continue;
      }
    }
#pragma unroll
    for (int q = 0; q < STEPS; ++q)
      store_split4<T>(r, n, (int64_t)h * dh, (int64_t)hh * dh + (g * STEPS + q) * 4, o[q], split);
  }
}

// TrainedSdm read (track4_onesdm_models.py:452-456): r[n, hh, :] = sum_j w[n, hh, j] * values[hh, si[n, hh, j], :]
// (embedding_bag, mode "sum", accumulated in float32 in j order).  One warp per (token, head).
template <typename T>
__global__ void ts_gather_kernel(const int32_t* __restrict__ si, const float* __restrict__ w,
                                 const T* __restrict__ values, int64_t N, int h, int M, int dh, int k,
                                 T* __restrict__ r, int split) {
  pdl_enter();
  int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  int lane = threadIdx.x & 31;
  if (item >= N * h) return;
  int hh = (int)(item % h);
  const int32_t* sr = si + item * k;
  const float* wr = w + item * k;
  for (int c0 = 0; c0 < dh; c0 += 256) {
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.f;
    for (int j = 0; j < k; ++j) {
      int slot = sr[j];
      float wj = wr[j];
      const T* row = values + ((int64_t)hh * M + slot) * dh;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        int c = c0 + lane + 32 * q;
        if (c < dh) acc[q] = fmaf(wj, to_f32(row[c]), acc[q]);
      }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      int c = c0 + lane + 32 * q;
      if (c < dh) store_split<T>(r, item / h, (int64_t)h * dh, hh * dh + c, acc[q], split);
    }
  }
}

// The same read for bf16 values with dh a multiple of 8 (at most 256) and k <= 32: lane l owns columns 8l..8l+7 and
// loads them as one 16-byte access per gathered row; the k (slot, weight) pairs are loaded once and broadcast.
__global__ void ts_gather_vec_kernel(const int32_t* __restrict__ si, const float* __restrict__ w,
                                     const bf16_t* __restrict__ values, int64_t N, int h, int M, int dh, int k,
                                     bf16_t* __restrict__ r, int split) {
  pdl_enter();
  const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (item >= N * h) return;
  const int hh = (int)(item % h);
  const int my_s = lane < k ? si[item * k + lane] : 0;
  const float my_w = lane < k ? w[item * k + lane] : 0.f;
  const bool active = 8 * lane < dh;
  const bf16_t* base = values + (int64_t)hh * M * dh + 8 * lane;
  float2 acc[4];  // columns (2q, 2q + 1) of the lane's eight
#pragma unroll
  for (int q = 0; q < 4; ++q) acc[q] = make_float2(0.f, 0.f);
  auto row = [&](int slot, float wj) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(base + (int64_t)slot * dh));  // read-only: L1 reuse
    const float2 w2 = make_float2(wj, wj);
    const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q)  // a bfloat16 pair widened exactly: the low half to the first float
      acc[q] = fma2(w2, make_float2(__uint_as_float(uw[q] << 16), __uint_as_float(uw[q] & 0xFFFF0000u)), acc[q]);
  };
  if ((k & 3) == 0 && ((reinterpret_cast<uintptr_t>(si + item * k) | reinterpret_cast<uintptr_t>(w + item * k)) & 15) == 0) {
    // four (slot, weight) pairs per pair of 16-byte loads, the same address on every lane (one L1 broadcast)
    const int4* s4 = reinterpret_cast<const int4*>(si + item * k);
    const float4* w4 = reinterpret_cast<const float4*>(w + item * k);
#pragma unroll 2
    for (int j = 0; j < k / 4; ++j) {
      const int4 ss = __ldg(s4 + j);
      const float4 ww = __ldg(w4 + j);
      if (active) {
        row(ss.x, ww.x);
        row(ss.y, ww.y);
        row(ss.z, ww.z);
        row(ss.w, ww.w);
      }
    }
  } else {
#pragma unroll 4
    for (int j = 0; j < k; ++j) {
      const int slot = __shfl_sync(0xffffffffu, my_s, j);
      const float wj = __shfl_sync(0xffffffffu, my_w, j);
      if (active) row(slot, wj);
    }
  }
  if (active) {
    const int64_t n = item / h, c = (int64_t)hh * dh + 8 * lane;
    store_split4<bf16_t>(r, n, (int64_t)h * dh, c, make_float4(acc[0].x, acc[0].y, acc[1].x, acc[1].y), split);
    store_split4<bf16_t>(r, n, (int64_t)h * dh, c + 4, make_float4(acc[2].x, acc[2].y, acc[3].x, acc[3].y), split);
  }
}

// Prefill gathers with every lane busy: an item's dh / 8 lanes (G, eight columns each) are packed back to back
// across the block (blockDim.x / G items per block, a warp may hold lanes of two items), where
// ts_gather_vec_kernel gives each item a whole warp and leaves 32 - G lanes idle (8 of 32 at dh = 192).  Each lane
// sums its eight columns over the item's k rows in slot order with the same fused multiply-adds, so the results are
// the same bit for bit.  Needs k % 4 == 0 and 16-byte aligned si, w and values.  Registers are capped for six
// 256-thread blocks per SM (40 instead of 52, a word spilled): more gathers in flight, 3.02 -> 2.83 ms per step.
__global__ void __launch_bounds__(256, 6) ts_gather_dense_kernel(const int32_t* __restrict__ si,
                                                              const float* __restrict__ w,
                                                              const bf16_t* __restrict__ values, int64_t N, int h,
                                                              int M, int dh, int k, bf16_t* __restrict__ r, int split) {
  pdl_enter();
  const int G = dh >> 3;
  const int il = (int)threadIdx.x / G, chunk = (int)threadIdx.x - il * G;
  const int64_t item = (int64_t)blockIdx.x * ((int)blockDim.x / G) + il;
  if (item >= N * h) return;
  const int hh = (int)(item % h);
  const bf16_t* base = values + (int64_t)hh * M * dh + 8 * chunk;
  float2 acc[4];  // columns (2q, 2q + 1) of the lane's eight
#pragma unroll
  for (int q = 0; q < 4; ++q) acc[q] = make_float2(0.f, 0.f);
  auto row = [&](int slot, float wj) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(base + (int64_t)slot * dh));  // read-only: L1 reuse
    const float2 w2 = make_float2(wj, wj);
    const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q)  // a bfloat16 pair widened exactly: the low half to the first float
      acc[q] = fma2(w2, make_float2(__uint_as_float(uw[q] << 16), __uint_as_float(uw[q] & 0xFFFF0000u)), acc[q]);
  };
  const int4* s4 = reinterpret_cast<const int4*>(si + item * k);
  const float4* w4 = reinterpret_cast<const float4*>(w + item * k);
#pragma unroll 2
  for (int j = 0; j < k / 4; ++j) {
    const int4 ss = __ldg(s4 + j);
    const float4 ww = __ldg(w4 + j);
    row(ss.x, ww.x);
    row(ss.y, ww.y);
    row(ss.z, ww.z);
    row(ss.w, ww.w);
  }
  const int64_t n = item / h, c = (int64_t)hh * dh + 8 * chunk;
  store_split4<bf16_t>(r, n, (int64_t)h * dh, c, make_float4(acc[0].x, acc[0].y, acc[1].x, acc[1].y), split);
  store_split4<bf16_t>(r, n, (int64_t)h * dh, c + 4, make_float4(acc[2].x, acc[2].y, acc[3].x, acc[3].y), split);
}

// Items per block of ts_gather_dense_kernel for G lanes per item: the fewest that fill whole warps, doubled while
// the block stays within 256 threads; 0 when G lanes of one item do not fit.
static int ts_dense_items(int G) {
  int ipb = 1;
  while ((G * ipb) % 32) ++ipb;
  if (G * ipb > 256) return 0;
  while (G * ipb * 2 <= 256) ipb *= 2;
  return ipb;
}

// Decode-sized gathers: a block of 8 warps takes 2 (token, head) items, each item's k rows split over 4 warps (k/4
// loads in flight per warp), the 4 partial rows summed in shared memory in warp order.
__global__ void __launch_bounds__(256) ts_gather_split_kernel(const int32_t* __restrict__ si,
                                                              const float* __restrict__ w,
                                                              const bf16_t* __restrict__ values, int64_t N, int h,
                                                              int M, int dh, int k, bf16_t* __restrict__ r, int split) {
  pdl_enter();
  __shared__ float part[8][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * 2 + (warp >> 2);
  const int sp = warp & 3;
  const bool live = item < N * h;
  const int hh = live ? (int)(item % h) : 0;
  const int jn = (k + 3) / 4, j0 = sp * jn, j1 = min(k, j0 + jn);
  const int my_s = live && j0 + lane < j1 ? si[item * k + j0 + lane] : 0;
  const float my_w = live && j0 + lane < j1 ? w[item * k + j0 + lane] : 0.f;
  const bool active = live && 8 * lane < dh;
  const bf16_t* base = values + (int64_t)hh * M * dh + 8 * lane;
  float acc[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) acc[q] = 0.f;
#pragma unroll 8
  for (int j = 0; j < j1 - j0; ++j) {
    const int slot = __shfl_sync(0xffffffffu, my_s, j);
    const float wj = __shfl_sync(0xffffffffu, my_w, j);
    if (active) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(base + (int64_t)slot * dh));
      const float4 a = unpack_bf16x4(make_uint2(u.x, u.y)), b = unpack_bf16x4(make_uint2(u.z, u.w));
      acc[0] = fmaf(wj, a.x, acc[0]);
      acc[1] = fmaf(wj, a.y, acc[1]);
      acc[2] = fmaf(wj, a.z, acc[2]);
      acc[3] = fmaf(wj, a.w, acc[3]);
      acc[4] = fmaf(wj, b.x, acc[4]);
      acc[5] = fmaf(wj, b.y, acc[5]);
      acc[6] = fmaf(wj, b.z, acc[6]);
      acc[7] = fmaf(wj, b.w, acc[7]);
    }
  }
  if (active) {
#pragma unroll
    for (int q = 0; q < 8; ++q) part[warp][8 * lane + q] = acc[q];
  }
  __syncthreads();
  if (sp == 0 && active) {
    float v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) v[q] = part[warp][8 * lane + q] + part[warp + 1][8 * lane + q] +
                                      part[warp + 2][8 * lane + q] + part[warp + 3][8 * lane + q];
    const int64_t n = item / h, c = (int64_t)hh * dh + 8 * lane;
    store_split4<bf16_t>(r, n, (int64_t)h * dh, c, make_float4(v[0], v[1], v[2], v[3]), split);
    store_split4<bf16_t>(r, n, (int64_t)h * dh, c + 4, make_float4(v[4], v[5], v[6], v[7]), split);
  }
}

// ------------------------------------------------------------------------------------------------- launchers
template <typename T>
cudaError_t launch_rmsnorm(const T* x, const T* w, int64_t rows, int d, float eps, T* y, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  LaunchScope scope_("rmsnorm", st);
  constexpr int E = 16 / sizeof(T);
  const bool al = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(y)) &
                   15) == 0;
  const int nch = d % (32 * E) == 0 ? d / (32 * E) : 0;
  if (al && nch >= 1 && nch <= 4) {
    const int wpb = rows < 148 * 8 ? 2 : 8;  // small launches: fewer warps per block, more SMs
    const unsigned grid = (unsigned)ceil_div(rows, wpb);
    switch (nch) {
      case 1: launch_k(rmsnorm_vec_kernel<T, 1>, dim3(grid), dim3(wpb * 32), 0, st, x, w, rows, eps, y); break;
      case 2: launch_k(rmsnorm_vec_kernel<T, 2>, dim3(grid), dim3(wpb * 32), 0, st, x, w, rows, eps, y); break;
      case 3: launch_k(rmsnorm_vec_kernel<T, 3>, dim3(grid), dim3(wpb * 32), 0, st, x, w, rows, eps, y); break;
      default: launch_k(rmsnorm_vec_kernel<T, 4>, dim3(grid), dim3(wpb * 32), 0, st, x, w, rows, eps, y); break;
    }
    return cudaGetLastError();
  }
  return launch_k(rmsnorm_kernel<T>, dim3((unsigned)ceil_div(rows, 8)), dim3(256), 0, st, x, w, rows, d, eps, y);
}
template <typename T>
cudaError_t launch_embed(const int32_t* ids, const T* emb, int64_t N, int d, int V, T* out, int* bad,
                         cudaStream_t st) {
  if (N == 0) return cudaSuccess;
  LaunchScope scope_("embed", st);
  return launch_k(embed_kernel<T>, dim3((unsigned)ceil_div(N, 8)), dim3(256), 0, st, ids, emb, N, d, V, out, bad);
}
template <typename T>
cudaError_t launch_swiglu_act(const T* gu, int64_t rows, int f, T* p, cudaStream_t st) {
  const int64_t n = rows * f;
  if (n == 0) return cudaSuccess;
  int64_t blocks = ceil_div(n, 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  LaunchScope scope_("swiglu_act", st);
  return launch_k(swiglu_act_kernel<T>, dim3((unsigned)blocks), dim3(256), 0, st, gu, rows, f, p);
}
template <typename T>
cudaError_t launch_rt_finish(const float* num, const float* den, int64_t N, int h, int dh, int read_sum,
                             float read_eps, int out_norm, float out_norm_eps, const float* onorm_w, T* r, int split,
                             cudaStream_t st) {
  if (N == 0) return cudaSuccess;
  LaunchScope scope_("rt_finish", st);
  const bool al = ((reinterpret_cast<uintptr_t>(num) | reinterpret_cast<uintptr_t>(onorm_w) |
                    reinterpret_cast<uintptr_t>(r)) & 15) == 0;
  if (al && (dh == 64 || dh == 32 || dh == 128)) {
    // rows per lane group: 4 while that still leaves at least two waves of 148 SMs x 8 blocks, else 1
    const bool big = N * h >= (int64_t)148 * 8 * 32 * 4 * 2;
    const int rows_per = big ? 4 : 1;
    const unsigned grid = (unsigned)ceil_div(ceil_div(N * h, rows_per) * 8, 256);
#define SDM_FIN(STEPS)                                                                                          \
  (big ? launch_k(rt_finish_vec_kernel<T, STEPS, 4>, dim3(grid), dim3(256), 0, st, num, den, N, h, read_sum,      \
                  read_eps, out_norm, out_norm_eps, onorm_w, r, split)                                          \
       : launch_k(rt_finish_vec_kernel<T, STEPS, 1>, dim3(grid), dim3(256), 0, st, num, den, N, h, read_sum,      \
                  read_eps, out_norm, out_norm_eps, onorm_w, r, split))
    if (dh == 64)
      SDM_FIN(2);
    else if (dh == 32)
      SDM_FIN(1);
    else
      SDM_FIN(4);
#undef SDM_FIN
    return cudaGetLastError();
  }
  return launch_k(rt_finish_kernel<T>, dim3((unsigned)ceil_div(N * h, 8)), dim3(256), 0, st, num, den, N, h, dh,
                  read_sum, read_eps, out_norm, out_norm_eps, onorm_w, r, split);
}
// TrainedSdm address + read for decode-sized launches (track4_onesdm_models.py:438-456), one block of four warps
// per (token, head): warps 0 and 1 build the two halves' sorted lists (each lane normalising and scoring its own
// sub-keys) while warp 2 lists the candidate pairs, warp 0 combines them (the warp-per-address selection of the
// addressing kernels, so the picks are identical) into shared memory and global memory (si, w), then the four
// warps gather the picked value rows as ts_gather_split_kernel does.  Saves the separate addressing launch of every
// decode step.
template <int HALF, int S>
__global__ void __launch_bounds__(128) ts_addr_gather_kernel(const float* __restrict__ q, int64_t ldq,
                                                             const float* __restrict__ keys1,
                                                             const float* __restrict__ keys2,
                                                             const float* __restrict__ log_scale, int n_sub, int d_a,
                                                             int kk, const bf16_t* __restrict__ values, int64_t N,
                                                             int h, int dh, int32_t* __restrict__ si,
                                                             float* __restrict__ w, bf16_t* __restrict__ r, int split) {
  pdl_enter();
  extern __shared__ float tsd_smem[];  // warp scratch (128), candidates (32 S)
  __shared__ float part[4][256];
  __shared__ int s_si[32];
  __shared__ float s_w[32];
  __shared__ int s_nc;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t item = blockIdx.x;
  const int hh = (int)(item % h);
  const int64_t n = item / h;
  float* wsm = tsd_smem;  // v1, i1, v2, i2
  int* cand = reinterpret_cast<int*>(tsd_smem + 128);
  const int c1 = kk < n_sub ? kk : n_sub;
  if (warp < 2) {  // the two halves' lists in parallel, each lane normalising its own sub-keys
    const bool zvec = HALF % 4 == 0 && ((reinterpret_cast<uintptr_t>(q) & 15) | (ldq & 3) | (d_a & 3)) == 0;
    const float* keys = (warp ? keys2 : keys1) + (int64_t)hh * n_sub * HALF;
    warp_half_list_own<HALF, S>(q + n * ldq + (int64_t)hh * d_a + warp * HALF, zvec, keys, n_sub, c1, wsm + warp * 64,
                                reinterpret_cast<int*>(wsm + warp * 64 + 32));
  } else if (warp == 2) {
    const int nc = warp_candidates(cand, c1, kk);
    if (lane == 0) s_nc = nc;
  }
  __syncthreads();
  if (warp == 0) {
    warp_combine<S>(wsm, n_sub, c1, kk, cand, s_nc, expf(log_scale[hh]), nullptr, s_si, s_w, nullptr);
    __syncwarp();
    if (lane < kk) {
      si[item * kk + lane] = s_si[lane];
      w[item * kk + lane] = s_w[lane];
    }
  }
  __syncthreads();
  const int jn = (kk + 3) / 4, j0 = warp * jn, j1 = min(kk, j0 + jn);
  const bool active = 8 * lane < dh;
  const bf16_t* base = values + (int64_t)hh * n_sub * n_sub * dh + 8 * lane;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  for (int j = j0; j < j1; ++j) {
    const int slot = s_si[j];
    const float wj = s_w[j];
    if (active) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(base + (int64_t)slot * dh));
      const float4 a = unpack_bf16x4(make_uint2(u.x, u.y)), b = unpack_bf16x4(make_uint2(u.z, u.w));
      acc[0] = fmaf(wj, a.x, acc[0]);
      acc[1] = fmaf(wj, a.y, acc[1]);
      acc[2] = fmaf(wj, a.z, acc[2]);
      acc[3] = fmaf(wj, a.w, acc[3]);
      acc[4] = fmaf(wj, b.x, acc[4]);
      acc[5] = fmaf(wj, b.y, acc[5]);
      acc[6] = fmaf(wj, b.z, acc[6]);
      acc[7] = fmaf(wj, b.w, acc[7]);
    }
  }
  if (active) {
#pragma unroll
    for (int e = 0; e < 8; ++e) part[warp][8 * lane + e] = acc[e];
  }
  __syncthreads();
  if (warp == 0 && active) {
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = part[0][8 * lane + e] + part[1][8 * lane + e] + part[2][8 * lane + e] +
                                      part[3][8 * lane + e];
    const int64_t c = (int64_t)hh * dh + 8 * lane;
    store_split4<bf16_t>(r, n, (int64_t)h * dh, c, make_float4(v[0], v[1], v[2], v[3]), split);
    store_split4<bf16_t>(r, n, (int64_t)h * dh, c + 4, make_float4(v[4], v[5], v[6], v[7]), split);
  }
}

bool ts_addr_gather_ok(int64_t N, int h, int d_a, int n_sub, int k, int dh) {
  const int c1 = k < n_sub ? k : n_sub, kk = k < c1 * c1 ? k : c1 * c1;
  return N * h < 148 * 8 && d_a == 32 && kk <= 32 && c1 <= 32 && dh % 8 == 0 && dh <= 256 &&
         pk_warp_slots(n_sub, c1, kk) > 0;
}

template <int S>
static cudaError_t launch_ts_addr_gather_s(const float* q, int64_t ldq, const float* keys1, const float* keys2,
                                           const float* log_scale, int n_sub, int kk, const bf16_t* values,
                                           int64_t N, int h, int dh, int32_t* si, float* w, bf16_t* r, int split,
                                           cudaStream_t st) {
  const size_t smem = ((size_t)128 + 32 * S) * 4;
  auto kern = ts_addr_gather_kernel<16, S>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_k(kern, dim3((unsigned)(N * h)), dim3(128), smem, st, q, ldq, keys1, keys2, log_scale, n_sub, 32, kk,
                  values, N, h, dh, si, w, r, split);
}

cudaError_t launch_ts_addr_gather(const float* q, int64_t ldq, const float* keys1, const float* keys2,
                                  const float* log_scale, int n_sub, int k, const bf16_t* values, int64_t N, int h,
                                  int dh, int32_t* si, float* w, bf16_t* r, int split, cudaStream_t st) {
  if (N == 0) return cudaSuccess;
  if (!ts_addr_gather_ok(N, h, 32, n_sub, k, dh) || (reinterpret_cast<uintptr_t>(values) & 15) != 0)
    return cudaErrorInvalidValue;
  const int c1 = k < n_sub ? k : n_sub, kk = k < c1 * c1 ? k : c1 * c1;
  LaunchScope scope_("ts_addr_gather", st);
  switch (pk_warp_slots(n_sub, c1, kk)) {
    case 1: return launch_ts_addr_gather_s<1>(q, ldq, keys1, keys2, log_scale, n_sub, kk, values, N, h, dh, si, w, r,
                                              split, st);
    case 2: return launch_ts_addr_gather_s<2>(q, ldq, keys1, keys2, log_scale, n_sub, kk, values, N, h, dh, si, w, r,
                                              split, st);
    default: return launch_ts_addr_gather_s<4>(q, ldq, keys1, keys2, log_scale, n_sub, kk, values, N, h, dh, si, w,
                                               r, split, st);
  }
}

template <typename T>
cudaError_t launch_ts_gather(const int32_t* si, const float* w, const T* values, int64_t N, int h, int M, int dh,
                             int k, T* r, int split, cudaStream_t st) {
  if (N == 0) return cudaSuccess;
  LaunchScope scope_("ts_gather", st);
  if constexpr (sizeof(T) == 2) {
    if (dh % 8 == 0 && dh <= 256 && k <= 32 && (reinterpret_cast<uintptr_t>(values) & 15) == 0) {
      if (N * h < 148 * 8) {  // decode-sized: spread each item's rows over four warps
        return launch_k(ts_gather_split_kernel, dim3((unsigned)ceil_div(N * h, 2)), dim3(256), 0, st, si, w, values,
                        N, h, M, dh, k, r, split);
      }
    }
    const int ipb = dh % 8 == 0 ? ts_dense_items(dh / 8) : 0;
    if (ipb > 0 && k % 4 == 0 && N * h >= 148 * 8 &&
        ((reinterpret_cast<uintptr_t>(si) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(values)) &
         15) == 0)
      return launch_k(ts_gather_dense_kernel, dim3((unsigned)ceil_div(N * h, ipb)), dim3((unsigned)(ipb * (dh / 8))),
                      0, st, si, w, values, N, h, M, dh, k, r, split);
    if (dh % 8 == 0 && dh <= 256 && k <= 32 && (reinterpret_cast<uintptr_t>(values) & 15) == 0)
      return launch_k(ts_gather_vec_kernel, dim3((unsigned)ceil_div(N * h, 8)), dim3(256), 0, st, si, w, values, N,
                      h, M, dh, k, r, split);
  }
  return launch_k(ts_gather_kernel<T>, dim3((unsigned)ceil_div(N * h, 8)), dim3(256), 0, st, si, w, values, N, h, M,
                  dh, k, r, split);
}

#define SDM_INST(T)                                                                                              \
  template cudaError_t launch_rmsnorm<T>(const T*, const T*, int64_t, int, float, T*, cudaStream_t);            \
  template cudaError_t launch_embed<T>(const int32_t*, const T*, int64_t, int, int, T*, int*, cudaStream_t);    \
  template cudaError_t launch_swiglu_act<T>(const T*, int64_t, int, T*, cudaStream_t);                          \
  template cudaError_t launch_rt_finish<T>(const float*, const float*, int64_t, int, int, int, float, int, float, \
                                           const float*, T*, int, cudaStream_t);                                 \
  template cudaError_t launch_ts_gather<T>(const int32_t*, const float*, const T*, int64_t, int, int, int, int, T*, \
                                           int, cudaStream_t);
SDM_INST(float)
SDM_INST(bf16_t)

}  // namespace sdm
