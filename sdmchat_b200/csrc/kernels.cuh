// Internal launch interface shared by the .cu files of libsdm_b200.
#pragma once
#include "common.cuh"

namespace sdm {

// ------------------------------------------------------------------------------------------- GEMM epilogues
// Each epilogue receives one accumulator element (row, col, acc) of y = x @ w^T and writes it.  `rows` and `n`
// bound the valid region; the GEMM kernels never call apply() outside it.

// Element-wise epilogues share one shape: column(col) returns what depends on the column only (hoisted out of the
// row loop by the tensor-core GEMM), load_input(row, col) fetches a per-element input when kHasInput (issued for 32
// rows at once before any is used), store(...) writes; apply(row, col, acc) composes them (the CUDA-core GEMM).
struct NoCol {};

// y (float32) = acc
struct EpiF32 {
  static constexpr bool kRowMode = false, kHasInput = false;
  float* y;
  int64_t ldy;
  using Col = NoCol;
  __device__ __forceinline__ Col column(int) const { return {}; }
  __device__ __forceinline__ float load_input(int64_t, int) const { return 0.f; }
  __device__ __forceinline__ void store(int64_t row, int col, float acc, const Col&, float) const {
    y[row * ldy + col] = acc;
  }
  __device__ __forceinline__ void apply(int64_t row, int col, float acc) const { store(row, col, acc, {}, 0.f); }
};
// y (float32) = acc rounded to the precision of T (logits of a bf16 head, then reduced in float32)
template <typename T>
struct EpiF32R {
  static constexpr bool kRowMode = false, kHasInput = false;
  float* y;
  int64_t ldy;
  using Col = NoCol;
  __device__ __forceinline__ Col column(int) const { return {}; }
  __device__ __forceinline__ float load_input(int64_t, int) const { return 0.f; }
  __device__ __forceinline__ void store(int64_t row, int col, float acc, const Col&, float) const {
    y[row * ldy + col] = round_to<T>(acc);
  }
  __device__ __forceinline__ void apply(int64_t row, int col, float acc) const { store(row, col, acc, {}, 0.f); }
};
// y (T) = round(acc)
template <typename T>
struct EpiStore {
  static constexpr bool kRowMode = false, kHasInput = false;
  T* y;
  int64_t ldy;
  using Col = NoCol;
  __device__ __forceinline__ Col column(int) const { return {}; }
  __device__ __forceinline__ float load_input(int64_t, int) const { return 0.f; }
  __device__ __forceinline__ void store(int64_t row, int col, float acc, const Col&, float) const {
    y[row * ldy + col] = from_f32<T>(acc);
  }
  __device__ __forceinline__ void apply(int64_t row, int col, float acc) const { store(row, col, acc, {}, 0.f); }
};
// RunTimeSdm.prepare's projection (track4_onesdm_models.py:199-205): columns [0, 2*h*d_a) are the write key and
// the read query, each + addr_b; [2*h*d_a, 2*h*d_a + d) the value; the last h columns the write gate
// sigmoid(acc + b).  Everything is stored float32 in one (rows, ldy) buffer.
struct EpiProj {
  static constexpr bool kRowMode = false, kHasInput = false;
  float* y;
  int64_t ldy;
  const float* addr_b;  // (h*d_a)
  const float* gate_b;  // (h)
  int hda;              // h*d_a
  int gate_from;        // 2*h*d_a + d
  struct Col {
    float bias;
    bool sig;
  };
  __device__ __forceinline__ Col column(int col) const {
    if (col < 2 * hda) return {addr_b[col < hda ? col : col - hda], false};
    if (col < gate_from) return {0.f, false};
    return {gate_b[col - gate_from], true};
  }
  __device__ __forceinline__ float load_input(int64_t, int) const { return 0.f; }
  __device__ __forceinline__ void store(int64_t row, int col, float acc, const Col& c, float) const {
    float v = acc + c.bias;
    if (c.sig) v = 1.f / (1.f + expf(-v));
    y[row * ldy + col] = v;
  }
  __device__ __forceinline__ void apply(int64_t row, int col, float acc) const {
    store(row, col, acc, column(col), 0.f);
  }
};
// Residual add of a module output (OneSdmLM.residual, track4_onesdm_models.py:540-547): the module output is
// rounded to T (its `.to(x.dtype)`), then x + out is rounded to T.  x == nullptr: y = round(acc).
template <typename T>
struct EpiResid {
  static constexpr bool kRowMode = false, kHasInput = true;
  const T* x;
  T* y;
  int64_t ld;
  using Col = NoCol;
  __device__ __forceinline__ Col column(int) const { return {}; }
  __device__ __forceinline__ float load_input(int64_t row, int col) const {
    return x ? to_f32(x[row * ld + col]) : 0.f;
  }
  __device__ __forceinline__ void store(int64_t row, int col, float acc, const Col&, float in) const {
    float o = round_to<T>(acc);
    if (x) o = in + o;
    y[row * ld + col] = from_f32<T>(o);
  }
  __device__ __forceinline__ void apply(int64_t row, int col, float acc) const {
    store(row, col, acc, {}, load_input(row, col));
  }
};

// Row-owned epilogues of the tied head (the tensor-core GEMM only): each epilogue thread owns one row of a
// 128-column tile and reduces it in registers.  Logits are rounded to bfloat16 first, as the bf16 head stores them.
// EpiCE: online logsumexp per (row, column tile) -> part[row * tiles_n + tile] = (max, sum exp(x - max)); the
// target's logit -> tgt_logit[row].  ce_combine folds the partials into the summed cross-entropy.
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
    float v[32];
    float cmax = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      v[j] = col0 + j < n ? bf16_round(__uint_as_float(r[j])) : -INFINITY;
      cmax = fmaxf(cmax, v[j]);
    }
    const float mn = fmaxf(rs.m, cmax);
    float s = rs.m == -INFINITY ? 0.f : rs.s * expf(rs.m - mn);
#pragma unroll
    for (int j = 0; j < 32; ++j) s += v[j] == -INFINITY ? 0.f : expf(v[j] - mn);
    rs.m = mn;
    rs.s = s;
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
// The tensor-core GEMM directly (row-owned epilogues have no CUDA-core path).
template <typename Epi>
cudaError_t launch_gemm_tc(const bf16_t* x, int64_t ldx, const bf16_t* w, int64_t ldw, int64_t rows, int K, int n,
                           Epi epi, cudaStream_t st, int kwrap);
constexpr int TC_BN = 128;  // column tile of the tensor-core GEMM (partials per row = ceil(n / TC_BN))
cudaError_t launch_ce_combine(const float2* part, const float* tgt_logit, const int32_t* targets, int64_t rows,
                              int tiles_n, double* loss_sum, cudaStream_t st);
cudaError_t launch_argmax_combine(const float2* part, int64_t rows, int tiles_n, int32_t* ids, cudaStream_t st);

// Generic GEMM y = x @ w^T; x (rows, K) row-major (ldx), w (n, K) row-major (ldw) (nn.Linear weight layout).
// kwrap (0 = K): w's K index is taken modulo kwrap, so x = [hi | lo] (K = 2*kwrap) against one w computes
// hi @ w^T + lo @ w^T -- the float32-accurate product of a value split into two bfloat16 halves.
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
template <typename T>
cudaError_t launch_swiglu_act(const T* g, const T* u, int64_t n, T* p, cudaStream_t st);
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
};
cudaError_t launch_pk_address(const PkArgs& a, cudaStream_t st);

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
};
cudaError_t launch_rt_scan(const ScanArgs& a, cudaStream_t st);
bool rt_scan_supported(int M, int dh, int k);
size_t rt_scan_workspace_bytes(int B, int T, int h, int k);

// Single-token decode on the lazily-decayed state.
struct DecodeArgs {
  const int32_t* siw; const float* ww; const int32_t* sir; const float* wr;  // (S, h, k)
  const float* V; int64_t ldv;                                             // (S, ldv)
  const float* decay; const uint8_t* reset;
  int S, h, M, dh, k;
  float* mem; float* cnt; float* scale; int32_t* last_w;
  float* num; float* den;  // (S, h, dh), (S, h)
};
cudaError_t launch_rt_decode(const DecodeArgs& a, cudaStream_t st);

// Tied-head loss / argmax reductions over a materialised logits block (rows, V) float32.
cudaError_t launch_ce_rows(const float* logits, int64_t rows, int V, const int32_t* targets, double* loss_sum,
                           cudaStream_t st);
cudaError_t launch_argmax_rows(const float* logits, int64_t rows, int V, int32_t* ids, cudaStream_t st);

}  // namespace sdm
