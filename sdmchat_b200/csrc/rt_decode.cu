// Single-token decode on the carried run-time memory state (new API: the reference has no carried-state decode;
// its recurrence RunTimeSdm.forward_sequential, track4_onesdm_models.py:285-299, is the oracle step by step),
// fused with RunTimeSdm.finish up to wo (:243-246: mean read, per-head RMS out-norm).
//
// The state of each (stream, head) lives in HBM as (mem, cnt, scale): the true state is scale * (mem, cnt).
// A step reads k rows (before the write, as the reference does), then applies the fade lazily: scale <- scale*lam
// and the k written rows get ww * v / scale.  So a step touches 2k rows instead of decaying all M rows.  When
// scale falls below 2^-60 the head's state is renormalised once (one pass, amortised over >= 1/log2(1/lam)*60
// steps).  Fade 0 is special: the state after a write is exactly that write, so the rows written at the previous
// step (last_w) are cleared instead.
//
// One CTA per (stream, head); thread c owns value column c (thread 0 also the slot counts and the per-head words).
// The step's slot ids and weights are staged in shared memory, then every row the step touches (k read rows, k
// written rows) is loaded in one round trip before any store; the read is finished in the block (one block
// reduction for the out-norm) and written as the wo GEMM's input.
#include "pk_common.cuh"

namespace sdm {

constexpr int DEC_MAX_K = 32;

// The address rows are read four floats at a time when their layout allows it.
template <int HALF>
__device__ __forceinline__ bool dec_zvec(const DecodeArgs& a) {
  return HALF % 4 == 0 &&
         ((reinterpret_cast<uintptr_t>(a.proj) & 15) | (a.ldp & 3) | (a.d_a & 3) | (a.h * a.d_a & 3)) == 0;
}


// HALF > 0: the step selects its slots itself (warps 0-3 the halves of the write and read addresses with SH sub-keys
// per lane, warps 0 and 2 the combines with S candidates per lane; shared-memory normalised sub-keys); HALF == 0:
// the selections come in siw/ww/sir/wr.  KM bounds k at
// compile time: the touched rows are held in registers (four KM-long arrays), and KM 16 (for k <= 16) keeps the
// block at about half the registers of KM 32, so twice as many (stream, head) blocks are resident.
// LBT, LBM: launch bounds (threads, resident blocks per SM); 128 threads x 8 blocks caps the register use at 64 (a few
// spilled words) so that eight (stream, head) blocks share an SM instead of five.
template <typename T, int HALF, int S, int SH, int KM, int LBT = 1024, int LBM = 1>
__global__ void __launch_bounds__(LBT, LBM) rt_decode_kernel(DecodeArgs a) {
  pdl_enter();
  __shared__ int s_ir[DEC_MAX_K], s_iw[DEC_MAX_K], s_prev[DEC_MAX_K];
  __shared__ float s_fr[DEC_MAX_K], s_fw[DEC_MAX_K], s_red[32];
  __shared__ int s_nc;
  extern __shared__ float dec_smem[];  // HALF > 0: sub-keys (2 x n_sub x HALF), two warps' scratch, candidates
  const int sh = blockIdx.x;
  const int hh = sh % a.h;
  const int s = sh / a.h;
  const int M = a.M, dh = a.dh, k = a.k;
  float* mem = a.mem + (int64_t)sh * M * dh;
  float* cnt = a.cnt + (int64_t)sh * M;
  int32_t* lw = a.last_w + (int64_t)sh * k;
  const int t = threadIdx.x, warp = t >> 5;
  // inputs read only at the end (the value column written, the out-norm weight), fetched first
  const float vc = t < dh ? a.V[(int64_t)s * a.ldv + (int64_t)hh * dh + t] : 0.f;
  const float onw = (t < dh && a.out_norm) ? a.onorm_w[hh * dh + t] : 1.f;
  if constexpr (HALF > 0) {
    const int n_sub = a.n_sub, c1 = min(a.k, n_sub);
    float* kn = dec_smem;
    if constexpr (SH > 1) {
      for (int j = t; j < 2 * n_sub; j += blockDim.x) {  // F.normalize(keys, dim=-1) for this head
        const float* src = (j < n_sub ? a.keys1 + ((int64_t)hh * n_sub + j) * HALF
                                      : a.keys2 + ((int64_t)hh * n_sub + (j - n_sub)) * HALF);
        float kv[HALF];
        normalize_half<HALF>(src, kv);
#pragma unroll
        for (int dd = 0; dd < HALF; ++dd) kn[j * HALF + dd] = kv[dd];
      }
    }
    if (warp == 0) {
      const int nc = warp_candidates(reinterpret_cast<int*>(kn + 2 * n_sub * HALF + 2 * 128), c1, k);
      if (t == 0) s_nc = nc;
    }
    if constexpr (SH == 1) {
      // n_sub <= 32: warps 0-3 build the (write keys, read queries) x (first, second half) lists at once, lane j
      // normalising sub-key j itself, with no barrier before them
      if (warp < 4) {
        const int ad = warp >> 1, hf = warp & 1;
        float* wsm = dec_smem + 2 * n_sub * HALF + ad * 128;  // per address: v1, i1, v2, i2
        const float* zh = a.proj + (int64_t)s * a.ldp + (ad ? a.h * a.d_a : 0) + hh * a.d_a + hf * HALF;
        const float* keys = (hf ? a.keys2 : a.keys1) + (int64_t)hh * n_sub * HALF;
        warp_half_list_own<HALF, 1, false>(zh, dec_zvec<HALF>(a), keys, n_sub, c1, wsm + hf * 64,
                                 reinterpret_cast<int*>(wsm + hf * 64 + 32));
      }
    }
  } else if (t < k) {  // slot ids are clamped into the state (see rt_scan.cu)
    s_ir[t] = min(max(a.sir[(int64_t)sh * k + t], 0), M - 1);
    s_fr[t] = a.wr[(int64_t)sh * k + t];
    s_iw[t] = min(max(a.siw[(int64_t)sh * k + t], 0), M - 1);
    s_fw[t] = a.ww[(int64_t)sh * k + t];
  }
  if (t < k) s_prev[t] = lw[t];
  const float lam = a.decay[hh];
  // every thread reads the per-head words (scale, last written rows) before thread 0 rewrites them
  const float sc = a.scale[sh];
  const bool reset = a.reset && a.reset[s];
  __syncthreads();
  if constexpr (HALF > 0) {
    // then warps 0 and 2 combine the halves of the write and the read address
    const int n_sub = a.n_sub, c1 = min(a.k, n_sub);
    float* wsm = dec_smem + 2 * n_sub * HALF + (warp >> 1) * 128;
    if constexpr (SH > 1) {
      if (warp < 4) {
        const int ad = warp >> 1, hf = warp & 1;
        const float* zh = a.proj + (int64_t)s * a.ldp + (ad ? a.h * a.d_a : 0) + hh * a.d_a + hf * HALF;
        warp_half_list<HALF, SH>(zh, dec_zvec<HALF>(a), dec_smem + hf * n_sub * HALF, n_sub, c1, wsm + hf * 64,
                                 reinterpret_cast<int*>(wsm + hf * 64 + 32));
      }
      __syncthreads();
    }
    if (warp == 0 || warp == 2) {
      const float* gate = (warp == 0 && a.gate_col >= 0) ? a.proj + (int64_t)s * a.ldp + a.gate_col + hh : nullptr;
      warp_combine<S>(wsm, n_sub, c1, k, reinterpret_cast<const int*>(dec_smem + 2 * n_sub * HALF + 2 * 128), s_nc,
                      expf(a.log_scale[hh]), gate, warp ? s_ir : s_iw, warp ? s_fr : s_fw, nullptr);
    }
    __syncthreads();
  }
  const int c = t;
  const bool act = c < dh;
  const bool own_cnt = (c == 0);
  const bool keep_old = lam != 0.f && !reset;
  // every row this step touches, loaded before the first store: the k read rows (each thread also loads the read
  // rows' counts, a warp-uniform broadcast, for the denominator) and the k written rows
  float rv[KM], rc[KM], wv[KM], wc[KM];
#pragma unroll
  for (int i = 0; i < KM; ++i) {
    if (i < k) {
      const int r = s_ir[i], q = s_iw[i];
      rv[i] = (act && !reset) ? mem[(int64_t)r * dh + c] : 0.f;
      rc[i] = reset ? 0.f : cnt[r];
      wv[i] = (act && keep_old) ? mem[(int64_t)q * dh + c] : 0.f;
      wc[i] = (own_cnt && keep_old) ? cnt[q] : 0.f;
    }
  }
  const float scr = reset ? 1.f : sc;
  float acc = 0.f, accd = 0.f;
#pragma unroll
  for (int i = 0; i < KM; ++i) {
    if (i < k) {
      acc = fmaf(s_fr[i], rv[i], acc);
      accd = fmaf(s_fr[i], rc[i], accd);
    }
  }
  // finish: mean (or sum) read, RMS over the head's dh columns, onorm_w
  float v = acc * scr;
  if (!a.read_sum) v = __fdiv_rn(v, accd * scr + a.read_eps);
  float ss = act ? v * v : 0.f;
  ss = warp_sum(ss);
  if ((t & 31) == 0) s_red[t >> 5] = ss;
  __syncthreads();  // also: every thread's loads of the state are done before the first store below
  if (act) {
    float tot = 0.f;
    for (int w = 0; w < (int)((blockDim.x + 31) >> 5); ++w) tot += s_red[w];
    const float rs = a.out_norm ? rsqrt_rn(__fdiv_rn(tot, (float)dh) + a.out_norm_eps) : 1.f;
    float o = v;
    if (a.out_norm) o = (o * rs) * onw;
    const int64_t d = (int64_t)a.h * dh, col = (int64_t)hh * dh + c;
    T* r = static_cast<T*>(a.r);
    if (a.split) {
      const float hi = round_to<T>(o);
      r[s * 2 * d + col] = from_f32<T>(hi);
      r[s * 2 * d + d + col] = from_f32<T>(o - hi);
    } else {
      r[s * d + col] = from_f32<T>(o);
    }
  }
  if (reset && act) {
    for (int r = 0; r < M; ++r) mem[(int64_t)r * dh + c] = 0.f;
    if (own_cnt)
      for (int r = 0; r < M; ++r) cnt[r] = 0.f;
  }
  float ns;
  if (lam == 0.f) {
    if (!reset && act) {
#pragma unroll
      for (int j = 0; j < KM; ++j) {
        if (j < k) {
          const int r = s_prev[j];
          if (r >= 0 && r < M) {
            mem[(int64_t)r * dh + c] = 0.f;
            if (own_cnt) cnt[r] = 0.f;
          }
        }
      }
    }
    ns = 1.f;
  } else {
    ns = scr * lam;
    if (ns < 8.673617e-19f) {  // 2^-60: fold the scale into the state (the written rows' loaded values too)
      if (act) {
        for (int r = 0; r < M; ++r) mem[(int64_t)r * dh + c] *= ns;
        if (own_cnt)
          for (int r = 0; r < M; ++r) cnt[r] *= ns;
      }
#pragma unroll
      for (int j = 0; j < KM; ++j) {
        if (j < k) {
          wv[j] *= ns;
          wc[j] *= ns;
        }
      }
      ns = 1.f;
    }
  }
  // write: state <- lam * state + sum_j ww_j (e_{siw_j} v^T, e_{siw_j}); the k written rows are distinct (a
  // top-k).  With fade 0 (or after a reset) every row not cleared above is zero, so the written value is the write.
  if (act) {
#pragma unroll
    for (int j = 0; j < KM; ++j) {
      if (j < k) {
        const int r = s_iw[j];
        const float f = __fdiv_rn(s_fw[j], ns);
        mem[(int64_t)r * dh + c] = fmaf(f, vc, wv[j]);
        if (own_cnt) cnt[r] = wc[j] + f;
      }
    }
  }
  if (own_cnt) {
    a.scale[sh] = ns;
    for (int j = 0; j < k; ++j) lw[j] = s_iw[j];
  }
}

bool rt_decode_fused_ok(int d_a, int n_sub, int k) {
  const int c1 = k < n_sub ? k : n_sub, kk = k < c1 * c1 ? k : c1 * c1;
  return d_a == 32 && k <= DEC_MAX_K && c1 <= 32 && kk <= 32 && pk_warp_slots(n_sub, c1, kk) > 0;
}

template <typename T, int S, int SH, int KM>
static cudaError_t launch_rt_decode_fused(const DecodeArgs& a, int threads, cudaStream_t st) {
  const size_t smem = ((size_t)2 * a.n_sub * 16 + 2 * 128 + 32 * S) * 4;
  void (*kern)(DecodeArgs) = rt_decode_kernel<T, 16, S, SH, KM>;
  if constexpr (KM == 16)
    if (threads == 128) kern = rt_decode_kernel<T, 16, S, SH, KM, 128, 8>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_k(kern, dim3((unsigned)((int64_t)a.S * a.h)), dim3(threads), smem, st, a);
}
template <typename T, int KM>
static cudaError_t launch_rt_decode_km(const DecodeArgs& a, cudaStream_t st) {
  if (a.keys1) {  // one thread per value column, and at least the four address warps
    if (!rt_decode_fused_ok(a.d_a, a.n_sub, a.k)) return cudaErrorInvalidValue;
    const int threads = a.dh > 128 ? ((a.dh + 31) / 32) * 32 : 128;
    // S: candidate pairs (and sub-keys) per lane of the combine; the half lists sort n_sub keys, one per lane when
    // n_sub <= 32 (a 32-key sort instead of the combine's 64 or 128)
    const bool one = a.n_sub <= 32;
    switch (pk_warp_slots(a.n_sub, a.k < a.n_sub ? a.k : a.n_sub, a.k)) {
      case 1: return launch_rt_decode_fused<T, 1, 1, KM>(a, threads, st);
      case 2: return one ? launch_rt_decode_fused<T, 2, 1, KM>(a, threads, st)
                         : launch_rt_decode_fused<T, 2, 2, KM>(a, threads, st);
      default: return one ? launch_rt_decode_fused<T, 4, 1, KM>(a, threads, st)
                          : launch_rt_decode_fused<T, 4, 4, KM>(a, threads, st);
    }
  }
  const int threads = ((a.dh + 31) / 32) * 32;  // one thread per value column
  return launch_k(rt_decode_kernel<T, 0, 1, 1, KM>, dim3((unsigned)((int64_t)a.S * a.h)), dim3(threads), 0, st, a);
}

template <typename T>
cudaError_t launch_rt_decode(const DecodeArgs& a, cudaStream_t st) {
  if (a.S == 0) return cudaSuccess;
  if (a.k > DEC_MAX_K || a.dh > 1024) return cudaErrorInvalidValue;
  LaunchScope scope_("rt_decode", st);
  if (a.k <= 16) return launch_rt_decode_km<T, 16>(a, st);
  return launch_rt_decode_km<T, DEC_MAX_K>(a, st);
}
template cudaError_t launch_rt_decode<float>(const DecodeArgs&, cudaStream_t);
template cudaError_t launch_rt_decode<bf16_t>(const DecodeArgs&, cudaStream_t);

// ----------------------------------------------------------------------------------------------- tied head
// Cross-entropy of one logits row (logsumexp - target logit), summed into a float64 total (ce_chunked's
// F.cross_entropy(..., reduction="sum"), track4_sdmllm24_fused_ce.py:76-77).  One block per row.
__global__ void ce_rows_kernel(const float* __restrict__ lg, int64_t rows, int V, const int32_t* __restrict__ tgt,
                               double* loss_sum) {
  pdl_enter();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int t = tgt[row];
  if (t < 0) return;
  const float* x = lg + row * V;
  float m = -INFINITY;
  for (int c = threadIdx.x; c < V; c += blockDim.x) m = fmaxf(m, x[c]);
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : -INFINITY;
    v = warp_max(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  m = red[0];
  __syncthreads();
  float s = 0.f;
  for (int c = threadIdx.x; c < V; c += blockDim.x) s += expf(x[c] - m);
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += red[w];
    const double lse = (double)m + log((double)tot);
    atomicAdd(loss_sum, lse - (double)x[t]);
  }
}

// argmax of one row, lowest index on ties.  One block per row.
__global__ void argmax_rows_kernel(const float* __restrict__ lg, int64_t rows, int V, int32_t* __restrict__ ids) {
  pdl_enter();
  __shared__ float rv[32];
  __shared__ int ri[32];
  const int64_t row = blockIdx.x;
  const float* x = lg + row * V;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = threadIdx.x; c < V; c += blockDim.x) {
    const float v = x[c];
    if (v > bv || (v == bv && c < bi)) {
      bv = v;
      bi = c;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    rv[threadIdx.x >> 5] = bv;
    ri[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    bv = rv[0];
    bi = ri[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
      if (rv[w] > bv || (rv[w] == bv && ri[w] < bi)) {
        bv = rv[w];
        bi = ri[w];
      }
    }
    ids[row] = bi;
  }
}

// Cross-entropy from the fused head's per-tile partials: per row, logsumexp = M + log(sum_i s_i exp(m_i - M)) over
// the column tiles, minus the target's logit; rows with target < 0 are skipped.  One warp per row, float64 total.
__global__ void ce_combine_kernel(const float2* __restrict__ part, const float* __restrict__ tgt_logit,
                                  const int32_t* __restrict__ targets, int64_t rows, int tiles_n, double* loss_sum) {
  pdl_enter();
  __shared__ double red[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  double contrib = 0.0;
  if (row < rows && targets[row] >= 0) {
    const float2* pr = part + row * tiles_n;
    float M = -INFINITY;
    for (int i = lane; i < tiles_n; i += 32) M = fmaxf(M, pr[i].x);
    M = warp_max(M);
    float S = 0.f;
    for (int i = lane; i < tiles_n; i += 32) {
      const float2 p = pr[i];
      if (p.x != -INFINITY) S += p.y * expf(p.x - M);
    }
    S = warp_sum(S);
    contrib = (double)M + log((double)S) - (double)tgt_logit[row];
  }
  if (lane == 0) red[warp] = contrib;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < 8; ++w) t += red[w];
    atomicAdd(loss_sum, t);
  }
}

// Greedy id from the fused head's per-tile (best, column) partials; lowest column on ties.  One warp per row.
__global__ void argmax_combine_kernel(const float2* __restrict__ part, int64_t rows, int tiles_n,
                                      int32_t* __restrict__ ids) {
  pdl_enter();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  if (row >= rows) return;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = lane; i < tiles_n; i += 32) {
    const float2 p = part[row * tiles_n + i];
    const int idx = __float_as_int(p.y);
    if (p.x > bv || (p.x == bv && idx < bi)) {
      bv = p.x;
      bi = idx;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) ids[row] = bi;
}

cudaError_t launch_ce_combine(const float2* part, const float* tgt_logit, const int32_t* targets, int64_t rows,
                              int tiles_n, double* loss_sum, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  LaunchScope scope_("ce_combine", st);
  return launch_k(ce_combine_kernel, dim3((unsigned)ceil_div(rows, 8)), dim3(256), 0, st, part, tgt_logit, targets,
                  rows, tiles_n, loss_sum);
}

cudaError_t launch_argmax_combine(const float2* part, int64_t rows, int tiles_n, int32_t* ids, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  LaunchScope scope_("argmax_combine", st);
  return launch_k(argmax_combine_kernel, dim3((unsigned)ceil_div(rows, 8)), dim3(256), 0, st, part, rows, tiles_n, ids);
}

cudaError_t launch_ce_rows(const float* logits, int64_t rows, int V, const int32_t* targets, double* loss_sum,
                           cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  LaunchScope scope_("ce_rows", st);
  return launch_k(ce_rows_kernel, dim3((unsigned)rows), dim3(256), 0, st, logits, rows, V, targets, loss_sum);
}
cudaError_t launch_argmax_rows(const float* logits, int64_t rows, int V, int32_t* ids, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  LaunchScope scope_("argmax_rows", st);
  return launch_k(argmax_rows_kernel, dim3((unsigned)rows), dim3(256), 0, st, logits, rows, V, ids);
}

}  // namespace sdm
