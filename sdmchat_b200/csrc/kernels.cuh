// Internal launch interface shared by the .cu files of libsdm_b200.
#pragma once
#include "common.cuh"

namespace sdm {

// ------------------------------------------------------------------------------------------- GEMM epilogues
// Each epilogue receives accumulator elements of y = x @ w^T and writes them; `rows` and `n` bound the valid region.
// Two call shapes:
//   apply(row, col, acc)              one element (the CUDA-core GEMMs);
//   prefetch(pre, rl0, rows, col, n)  + store4(pre, it, row, col, acc4, n): the tensor-core GEMM's epilogue thread
//     owns columns col .. col+3 of rows rl0 + 4*it (it < 8); prefetch fetches what those need from global memory
//     (biases, the residual input) before the accumulator is ready, store4 writes the four values (16-byte or
//     8-byte stores when aligned; a column tail past n is written element by element).
struct NoPre {};

__device__ __forceinline__ bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
__device__ __forceinline__ bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; }
__device__ __forceinline__ float f4get(const float4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}
__device__ __forceinline__ uint2 pack_bf16x4(float4 v) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
  return make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
}
__device__ __forceinline__ float4 unpack_bf16x4(uint2 u) {
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
// Four consecutive values of T at d (m = how many of them are valid, 1..4+).
__device__ __forceinline__ void store4_to(float* d, float4 v, int m) {
  if (m >= 4 && aligned16(d)) {
    *reinterpret_cast<float4*>(d) = v;
  } else {
    for (int i = 0; i < 4 && i < m; ++i) d[i] = f4get(v, i);
  }
}
__device__ __forceinline__ void store4_to(bf16_t* d, float4 v, int m) {
  if (m >= 4 && aligned8(d)) {
    *reinterpret_cast<uint2*>(d) = pack_bf16x4(v);
  } else {
    for (int i = 0; i < 4 && i < m; ++i) d[i] = __float2bfloat16_rn(f4get(v, i));
  }
}
__device__ __forceinline__ float4 load4_from(const float* s, int m) {
  if (m >= 4 && aligned16(s)) return *reinterpret_cast<const float4*>(s);
  float t[4] = {0.f, 0.f, 0.f, 0.f};
  for (int i = 0; i < 4 && i < m; ++i) t[i] = s[i];
  return make_float4(t[0], t[1], t[2], t[3]);
}
__device__ __forceinline__ float4 load4_from(const bf16_t* s, int m) {
  if (m >= 4 && aligned8(s)) return unpack_bf16x4(*reinterpret_cast<const uint2*>(s));
  float t[4] = {0.f, 0.f, 0.f, 0.f};
  for (int i = 0; i < 4 && i < m; ++i) t[i] = __bfloat162float(s[i]);
  return make_float4(t[0], t[1], t[2], t[3]);
}

// Four values of T as loaded from memory (bf16: 8 bytes), for prefetched inputs held in registers.
template <typename T>
struct Pack4;
template <>
struct Pack4<float> {
  using type = float4;
  __device__ __forceinline__ static float4 load(const float* s, int m) { return load4_from(s, m); }
  __device__ __forceinline__ static float4 zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
  __device__ __forceinline__ static float4 unpack(float4 v) { return v; }
};
template <>
struct Pack4<bf16_t> {
  using type = uint2;
  __device__ __forceinline__ static uint2 load(const bf16_t* s, int m) {
    if (m >= 4 && aligned8(s)) return *reinterpret_cast<const uint2*>(s);
    return pack_bf16x4(load4_from(s, m));  // exact: the values are bf16 already
  }
  __device__ __forceinline__ static uint2 zero() { return make_uint2(0u, 0u); }
  __device__ __forceinline__ static float4 unpack(uint2 u) { return unpack_bf16x4(u); }
};

// y (float32) = acc
struct EpiF32 {
  static constexpr bool kRowMode = false;
  float* y;
  int64_t ldy;
  using Pre = NoPre;
  __device__ __forceinline__ void apply(int64_t row, int col, float acc) const { y[row * ldy + col] = acc; }
  __device__ __forceinline__ void prefetch(Pre&, int64_t, int64_t, int, int) const {}
  __device__ __forceinline__ void store4(const Pre&, int, int64_t row, int col, float4 v, int n) const {
    store4_to(y + row * ldy + col, v, n - col);
  }
};
// y (float32) = acc rounded to the precision of T (logits of a bf16 head, then reduced in float32)
template <typename T>
struct EpiF32R {
  static constexpr bool kRowMode = false;
  float* y;
  int64_t ldy;
  using Pre = NoPre;
  __device__ __forceinline__ void apply(int64_t row, int col, float acc) const { y[row * ldy + col] = round_to<T>(acc); }
  __device__ __forceinline__ void prefetch(Pre&, int64_t, int64_t, int, int) const {}
  __device__ __forceinline__ void store4(const Pre&, int, int64_t row, int col, float4 v, int n) const {
    store4_to(y + row * ldy + col, make_float4(round_to<T>(v.x), round_to<T>(v.y), round_to<T>(v.z), round_to<T>(v.w)),
              n - col);
  }
};
// y (T) = round(acc)
template <typename T>
struct EpiStore {
  static constexpr bool kRowMode = false;
  T* y;
  int64_t ldy;
  using Pre = NoPre;
  __device__ __forceinline__ void apply(int64_t row, int col, float acc) const { y[row * ldy + col] = from_f32<T>(acc); }
  __device__ __forceinline__ void prefetch(Pre&, int64_t, int64_t, int, int) const {}
  __device__ __forceinline__ void store4(const Pre&, int, int64_t row, int col, float4 v, int n) const {
    store4_to(y + row * ldy + col, v, n - col);
  }
};
// RunTimeSdm.prepare's projection (track4_onesdm_models.py:199-205): columns [0, 2*h*d_a) are the write key and
// the read query, each + addr_b; [2*h*d_a, 2*h*d_a + d) the value; the last h columns the write gate
// sigmoid(acc + b).  Everything is stored float32 in one (rows, ldy) buffer.
struct EpiProj {
  static constexpr bool kRowMode = false;
  float* y;
  int64_t ldy;
  const float* addr_b;  // (h*d_a)
  const float* gate_b;  // (h)
  int hda;              // h*d_a
  int gate_from;        // 2*h*d_a + d
  __device__ __forceinline__ float bias(int col) const {
    if (col < 2 * hda) return addr_b[col < hda ? col : col - hda];
    return col < gate_from ? 0.f : gate_b[col - gate_from];
  }
  __device__ __forceinline__ static float finish(float acc, float b, bool sig) {
    const float v = acc + b;
    return sig ? 1.f / (1.f + expf(-v)) : v;
  }
  __device__ __forceinline__ void apply(int64_t row, int col, float acc) const {
    y[row * ldy + col] = finish(acc, bias(col), col >= gate_from);
  }
  struct Pre {
    float4 b;
  };
  __device__ __forceinline__ void prefetch(Pre& p, int64_t, int64_t, int col, int n) const {
    float t[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) t[i] = col + i < n ? bias(col + i) : 0.f;
    p.b = make_float4(t[0], t[1], t[2], t[3]);
  }
  __device__ __forceinline__ void store4(const Pre& p, int, int64_t row, int col, float4 v, int n) const {
    float4 o = make_float4(v.x + p.b.x, v.y + p.b.y, v.z + p.b.z, v.w + p.b.w);
    if (col + 3 >= gate_from) gate4(o, col);  // only the last h columns take the sigmoid
    store4_to(y + row * ldy + col, o, n - col);
  }
  __device__ __noinline__ void gate4(float4& o, int col) const {
    if (col >= gate_from) o.x = 1.f / (1.f + expf(-o.x));
    if (col + 1 >= gate_from) o.y = 1.f / (1.f + expf(-o.y));
    if (col + 2 >= gate_from) o.z = 1.f / (1.f + expf(-o.z));
    if (col + 3 >= gate_from) o.w = 1.f / (1.f + expf(-o.w));
  }
};
// Residual add of a module output (OneSdmLM.residual, track4_onesdm_models.py:540-547): the module output is
// rounded to T (its `.to(x.dtype)`), then x + out is rounded to T.  x == nullptr: y = round(acc).
template <typename T>
struct EpiResid {
  static constexpr bool kRowMode = false;
  const T* x;
  T* y;
  int64_t ld;
  __device__ __forceinline__ float out1(float acc, float in) const {
    const float o = round_to<T>(acc);
    return x ? in + o : o;
  }
  __device__ __forceinline__ void apply(int64_t row, int col, float acc) const {
    y[row * ld + col] = from_f32<T>(out1(acc, x ? to_f32(x[row * ld + col]) : 0.f));
  }
  struct Pre {
    typename Pack4<T>::type in[8];  // the residual input, packed as stored
  };
  __device__ __forceinline__ void prefetch(Pre& p, int64_t rl0, int64_t rows, int col, int n) const {
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int64_t row = rl0 + 4 * it;
      p.in[it] = (x && row < rows && col < n) ? Pack4<T>::load(x + row * ld + col, n - col) : Pack4<T>::zero();
    }
  }
  __device__ __forceinline__ void store4(const Pre& p, int it, int64_t row, int col, float4 v, int n) const {
    const float4 in = Pack4<T>::unpack(p.in[it]);
    store4_to(y + row * ld + col, make_float4(out1(v.x, in.x), out1(v.y, in.y), out1(v.z, in.z), out1(v.w, in.w)),
              n - col);
  }
};

// Row-owned epilogues of the tied head (the tensor-core GEMM only): each epilogue thread owns one row of a
// 128-column tile and reduces it in registers.  Logits are rounded to bfloat16 first, as the bf16 head stores them.
// EpiCE: online logsumexp per (row, column tile) -> part[row * tiles_n + tile] = (max, sum exp(x - max)); the
// target's logit -> tgt_logit[row].  ce_combine folds the partials into the summed cross-entropy.  The exponentials
// of the max-shifted logits (all <= 0) use the hardware exponential __expf (relative error about 1e-6 there), summed
// in four interleaved partial sums; the loss is a float64 sum of per-row terms, so this stays near 1e-7 relative.
struct EpiCE {
  static constexpr bool kRowMode = true;
  const int32_t* targets;
  float2* part;
  float* tgt_logit;
  struct RowState {
    float m, s, tv;
    int tgt;
    bool has;
  };
  __device__ __forceinline__ void row_begin(RowState& rs, int64_t row, int64_t rows, int) const {
    rs.m = -INFINITY;
    rs.s = 0.f;
    rs.tv = 0.f;
    rs.has = false;
    rs.tgt = row < rows ? targets[row] : -1;
  }
  __device__ __forceinline__ void row_chunk(RowState& rs, int col0, int n, const uint32_t (&r)[32]) const {
    if (col0 >= n) return;  // past the last column
    float v[32];
    if (col0 + 32 <= n) {
#pragma unroll
      for (int j = 0; j < 32; j += 2) {  // the logits rounded to bfloat16, two per conversion
        const __nv_bfloat162 p = __floats2bfloat162_rn(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
        v[j] = __low2float(p);
        v[j + 1] = __high2float(p);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = col0 + j < n ? bf16_round(__uint_as_float(r[j])) : -INFINITY;
    }
    float m4[4] = {v[0], v[1], v[2], v[3]};  // four independent chains, then a tree
#pragma unroll
    for (int j = 4; j < 32; ++j) m4[j & 3] = fmaxf(m4[j & 3], v[j]);
    const float cmax = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
    const float mn = fmaxf(rs.m, cmax);  // finite: column col0 is a real logit
    float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 32; ++j) s4[j & 3] += __expf(v[j] - mn);  // exp(-inf) = 0 for columns past n
    const float s = (s4[0] + s4[1]) + (s4[2] + s4[3]);
    rs.s = (rs.m == -INFINITY ? 0.f : rs.s * __expf(rs.m - mn)) + s;
    rs.m = mn;
    const int t = rs.tgt - col0;
    if (t >= 0 && t < 32) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j == t) rs.tv = v[j];
      rs.has = true;
    }
  }
  __device__ __forceinline__ void row_end(const RowState& rs, int64_t row, int64_t rows, int tn, int tiles_n) const {
    if (row >= rows) return;
    part[row * tiles_n + tn] = make_float2(rs.m, rs.s);
    if (rs.has) tgt_logit[row] = rs.tv;
  }
};
// EpiArgmax: greedy pick per (row, column tile) -> part[row * tiles_n + tile] = (best logit, its column), lowest
// column on ties; argmax_combine picks across tiles.
struct EpiArgmax {
  static constexpr bool kRowMode = true;
  float2* part;
  struct RowState {
    float best;
    int idx;
  };
  __device__ __forceinline__ void row_begin(RowState& rs, int64_t, int64_t, int) const {
    rs.best = -INFINITY;
    rs.idx = 0x7fffffff;
  }
  __device__ __forceinline__ void row_chunk(RowState& rs, int col0, int n, const uint32_t (&r)[32]) const {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float v = bf16_round(__uint_as_float(r[j]));
      if (col0 + j < n && v > rs.best) {
        rs.best = v;
        rs.idx = col0 + j;
      }
    }
  }
  __device__ __forceinline__ void row_end(const RowState& rs, int64_t row, int64_t rows, int tn, int tiles_n) const {
    if (row < rows) part[row * tiles_n + tn] = make_float2(rs.best, __int_as_float(rs.idx));
  }
};
// EpiSwiGLU: SwiGLU's gate and up maps (L:96-97) as one GEMM against the packed weight of swiglu_pack_rows: packed
// columns [32j, 32j + 16) are gate rows [16j, 16j + 16) and [32j + 16, 32j + 32) the up rows of the same f-indices,
// so one thread's 32-column chunk holds both factors of 16 outputs.  Each is rounded as the bfloat16 reference
// rounds: g and u (the Linear outputs), silu(g), then the product; only p = silu(g) * u reaches memory (bfloat16,
// (rows, f) with row stride ldp, 32-byte row segments).  silu(g) = g / (1 + e^-g) with the hardware exponential and
// division (a few 1e-7 relative before its bfloat16 rounding, which it changes only within that distance of a
// rounding boundary).
struct EpiSwiGLU {
  static constexpr bool kRowMode = true;
  bf16_t* p;
  int64_t ldp;
  struct RowState {
    int64_t row;
    bool live;
  };
  __device__ __forceinline__ void row_begin(RowState& rs, int64_t row, int64_t rows, int) const {
    rs.row = row;
    rs.live = row < rows;
  }
  __device__ __forceinline__ void row_chunk(RowState& rs, int col0, int n, const uint32_t (&r)[32]) const {
    if (!rs.live || col0 >= n) return;
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float v[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float g = bf16_round(__uint_as_float(r[2 * i + j]));
        const float u = bf16_round(__uint_as_float(r[16 + 2 * i + j]));
        v[j] = bf16_round(__fdividef(g, 1.f + __expf(-g))) * u;
      }
      const __nv_bfloat162 b2 = __floats2bfloat162_rn(v[0], v[1]);
      o[i] = *reinterpret_cast<const uint32_t*>(&b2);
    }
    uint4* dst = reinterpret_cast<uint4*>(p + rs.row * ldp + (col0 >> 1));
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
  __device__ __forceinline__ void row_end(const RowState&, int64_t, int64_t, int, int) const {}
};
// The tensor-core GEMM directly (row-owned epilogues have no CUDA-core path).
template <typename Epi>
cudaError_t launch_gemm_tc(const bf16_t* x, int64_t ldx, const bf16_t* w, int64_t ldw, int64_t rows, int K, int n,
                           Epi epi, cudaStream_t st, int kwrap);
constexpr int TC_BN = 128;  // columns per row-mode partial of the tensor-core GEMM (partials per row = ceil(n / 128))
cudaError_t launch_ce_combine(const float2* part, const float* tgt_logit, const int32_t* targets, int64_t rows,
                              int tiles_n, double* loss_sum, cudaStream_t st);
cudaError_t launch_argmax_combine(const float2* part, int64_t rows, int tiles_n, int32_t* ids, cudaStream_t st);

// Generic GEMM y = x @ w^T; x (rows, K) row-major (ldx), w (n, K) row-major (ldw) (nn.Linear weight layout).
// kwrap (0 = K): w's K index is taken modulo kwrap, so x = [hi | lo] (K = 2*kwrap) against one w computes
// hi @ w^T + lo @ w^T -- the product of a float32 value split into two bfloat16 parts (16 significant bits,
// within 2^-17 relative per element) with float32 accumulation.
// float: CUDA-core FMA; bf16: tcgen05 tensor cores when tc_gemm_supported(), else CUDA cores.
template <typename TA, typename Epi>
cudaError_t launch_gemm(const TA* x, int64_t ldx, const TA* w, int64_t ldw, int64_t rows, int K, int n, Epi epi,
                        cudaStream_t st, int kwrap = 0);
// Can the tensor-core GEMM take this shape (K a multiple of 64, 16-byte aligned rows and pointers)?
bool tc_gemm_supported(const void* x, int64_t ldx, const void* w, int64_t ldw, int K, int kwrap);

// ---------------------------------------------------------------------------------------------- other kernels
template <typename T>
cudaError_t launch_rmsnorm(const T* x, const T* w, int64_t rows, int d, float eps, T* y, cudaStream_t st);
template <typename T>
cudaError_t launch_embed(const int32_t* ids, const T* emb, int64_t N, int d, int V, T* out, int* bad,
                         cudaStream_t st);
// p (rows, f) = silu(gate) * up from the packed gate|up GEMM output gu (rows, 2f) (layout of EpiSwiGLU).
template <typename T>
cudaError_t launch_swiglu_act(const T* gu, int64_t rows, int f, T* p, cudaStream_t st);
// The module outputs below feed a wo GEMM whose reference input is float32: with split, row n of r holds the
// bfloat16 high part in columns [0, d) and the bfloat16 remainder in [d, 2d) (r is (N, 2d)); else r is (N, d).
template <typename T>
cudaError_t launch_rt_finish(const float* num, const float* den, int64_t N, int h, int dh, int read_sum,
                             float read_eps, int out_norm, float out_norm_eps, const float* onorm_w, T* r, int split,
                             cudaStream_t st);
template <typename T>
cudaError_t launch_ts_gather(const int32_t* si, const float* w, const T* values, int64_t N, int h, int M, int dh,
                             int k, T* r, int split, cudaStream_t st);

// Product-key addressing (track4_onesdm_models.py:134-148) with the soft weights of prepare (:203-206).
struct PkArgs {
  const float* z;       // address of token n, head hh at z[n * ldz + hh * d_a]
  int64_t ldz;
  const float* keys1;   // (h, n_sub, d_a/2)
  const float* keys2;
  int64_t N;            // tokens
  int h, d_a, n_sub, k;
  // outputs: with T_bh > 0 the (B, h, T, kk) layout of prepare (token n = b * T_bh + t), else (N, h, kk)
  int T_bh;
  float* sv;            // raw scores (or nullptr)
  float* w;             // softmax(scale * score) [* gate] (or nullptr)
  int32_t* si;          // slot ids
  const float* log_scale;  // (h), needed when w != nullptr
  const float* gate;    // gate of token n, head hh at gate[n * ldgate + hh] (or nullptr)
  int64_t ldgate;
  // pairs == 2: a second address set against the same sub-keys in the same launch (RunTimeSdm's write keys and
  // read queries): z2 / sv2 / w2 / si2 / gate2 play the roles of z / sv / w / si / gate
  int pairs;
  const float* z2;
  float* sv2;
  float* w2;
  int32_t* si2;
  const float* gate2;
};
cudaError_t launch_pk_address(const PkArgs& a, cudaStream_t st);
// TrainedSdm selection + value read in one launch for decode-sized calls (N * h below 1,184, d_a 32, bf16 values):
// q (N, ldq) float32 queries -> si, w (N, h, kk) and the read r (hi/lo split rows when split).
bool ts_addr_gather_ok(int64_t N, int h, int d_a, int n_sub, int k, int dh);
cudaError_t launch_ts_addr_gather(const float* q, int64_t ldq, const float* keys1, const float* keys2,
                                  const float* log_scale, int n_sub, int k, const bf16_t* values, int64_t N, int h,
                                  int dh, int32_t* si, float* w, bf16_t* r, int split, cudaStream_t st);

// The chunked write-then-read scan of RunTimeSdm (track4_onesdm_models.py:215-241, 255-272): a parallel pass per
// (row, head, chunk) that builds the chunk's slot lists and its intra-chunk reads, then the state scan.
struct ScanArgs {
  const int32_t* siw; const float* ww; const int32_t* sir; const float* wr;  // (B, h, T, k)
  const float* V; int64_t ldv;                                             // (B*T, ldv), head hh at hh*dh
  const float* decay; const uint8_t* reset;
  int B, T, h, M, dh, k;
  float* num;   // (B*T, h, dh)
  float* den;   // (B*T, h)
  float* mem_out; float* cnt_out;
  unsigned char* rec;  // chunk records, rt_scan_workspace_bytes(B, T, h, k) bytes
  // the state carried in (RunTimeSdm._chunk's mem, cnt: (B, h, M, dh), (B, h, M)), or both nullptr for an empty one
  const float* mem_in; const float* cnt_in;
};
cudaError_t launch_rt_scan(const ScanArgs& a, cudaStream_t st);
bool rt_scan_supported(int M, int dh, int k);
size_t rt_scan_workspace_bytes(int B, int T, int h, int k);
cudaError_t read_and_clear_scan_timeout(int* flag, cudaStream_t st);
// Bounded-wait limits of the scan and GEMM modules (0 = the default, about 4 s), and the wait probe.
cudaError_t set_scan_wait_limit(unsigned long long ns);
cudaError_t set_gemm_wait_limit(unsigned long long ns);
cudaError_t launch_wait_probe(int* done, cudaStream_t st);

// Single-token decode on the lazily-decayed state.
struct DecodeArgs {
  const int32_t* siw; const float* ww; const int32_t* sir; const float* wr;  // (S, h, k)
  const float* V; int64_t ldv;                                             // (S, ldv)
  const float* decay; const uint8_t* reset;
  int S, h, M, dh, k;
  float* mem; float* cnt; float* scale; int32_t* last_w;
  // RunTimeSdm.finish up to wo, fused: r (S, h * dh) in T (hi/lo bfloat16 rows (S, 2, h * dh) when split)
  int read_sum; float read_eps; int out_norm; float out_norm_eps; const float* onorm_w;
  void* r; int split;
  // addressing inside the step (keys1 != nullptr; then siw/ww/sir/wr are unused): the projection row of stream s
  // holds the write keys at proj[s * ldp + hh * d_a], the read queries h * d_a further, the gate at column
  // gate_col + hh (gate_col < 0: no write gate)
  const float* proj; int64_t ldp; const float* keys1; const float* keys2; const float* log_scale;
  int n_sub, d_a, gate_col;
};
// True when the decode step can select its slots itself (d_a 32 and a warp-sized selection).
bool rt_decode_fused_ok(int d_a, int n_sub, int k);
template <typename T>
cudaError_t launch_rt_decode(const DecodeArgs& a, cudaStream_t st);

// Tied-head loss / argmax reductions over a materialised logits block (rows, V) float32.
cudaError_t launch_ce_rows(const float* logits, int64_t rows, int V, const int32_t* targets, double* loss_sum,
                           cudaStream_t st);
cudaError_t launch_argmax_rows(const float* logits, int64_t rows, int V, int32_t* ids, cudaStream_t st);

}  // namespace sdm
