// Internal launch interface shared by the .cu files of libsdm_b200.
#pragma once
#include "common.cuh"

namespace sdm {

// ------------------------------------------------------------------------------------------- GEMM epilogues
// Each epilogue receives one accumulator element (row, col, acc) of y = x @ w^T and writes it.  `rows` and `n`
// bound the valid region; the GEMM kernels never call apply() outside it.

// y (float32) = acc
struct EpiF32 {
  float* y;
  int64_t ldy;
  __device__ __forceinline__ void apply(int64_t row, int col, float acc) const { y[row * ldy + col] = acc; }
};
// y (float32) = acc rounded to the precision of T (logits of a bf16 head, then reduced in float32)
template <typename T>
struct EpiF32R {
  float* y;
  int64_t ldy;
  __device__ __forceinline__ void apply(int64_t row, int col, float acc) const {
    y[row * ldy + col] = round_to<T>(acc);
  }
};
// y (T) = round(acc)
template <typename T>
struct EpiStore {
  T* y;
  int64_t ldy;
  __device__ __forceinline__ void apply(int64_t row, int col, float acc) const {
    y[row * ldy + col] = from_f32<T>(acc);
  }
};
// RunTimeSdm.prepare's projection (track4_onesdm_models.py:199-205): columns [0, 2*h*d_a) are the write key and
// the read query, each + addr_b; [2*h*d_a, 2*h*d_a + d) the value; the last h columns the write gate
// sigmoid(acc + b).  Everything is stored float32 in one (rows, ldy) buffer.
struct EpiProj {
  float* y;
  int64_t ldy;
  const float* addr_b;  // (h*d_a)
  const float* gate_b;  // (h)
  int hda;              // h*d_a
  int gate_from;        // 2*h*d_a + d
  __device__ __forceinline__ void apply(int64_t row, int col, float acc) const {
    float v;
    if (col < 2 * hda) {
      v = acc + addr_b[col < hda ? col : col - hda];
    } else if (col < gate_from) {
      v = acc;
    } else {
      float g = acc + gate_b[col - gate_from];
      v = 1.f / (1.f + expf(-g));
    }
    y[row * ldy + col] = v;
  }
};
// Residual add of a module output (OneSdmLM.residual, track4_onesdm_models.py:540-547): the module output is
// rounded to T (its `.to(x.dtype)`), then x + out is rounded to T.  x == nullptr: y = round(acc).
template <typename T>
struct EpiResid {
  const T* x;
  T* y;
  int64_t ld;
  __device__ __forceinline__ void apply(int64_t row, int col, float acc) const {
    float o = round_to<T>(acc);
    if (x) o = to_f32(x[row * ld + col]) + o;
    y[row * ld + col] = from_f32<T>(o);
  }
};

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

// The chunked write-then-read scan of RunTimeSdm (track4_onesdm_models.py:215-241, 255-272).
struct ScanArgs {
  const int32_t* siw; const float* ww; const int32_t* sir; const float* wr;  // (B, h, T, k)
  const float* V; int64_t ldv;                                             // (B*T, ldv), head hh at hh*dh
  const float* decay; const uint8_t* reset;
  int B, T, h, M, dh, k;
  float* num;   // (B*T, h, dh)
  float* den;   // (B*T, h)
  float* mem_out; float* cnt_out;
};
cudaError_t launch_rt_scan(const ScanArgs& a, cudaStream_t st);
bool rt_scan_supported(int M, int dh, int k);

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
