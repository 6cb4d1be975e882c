// Single-token decode on the carried run-time memory state (new API: the reference has no carried-state decode;
// its recurrence RunTimeSdm.forward_sequential, track4_onesdm_models.py:285-299, is the oracle step by step).
//
// The state of each (stream, head) lives in HBM as (mem, cnt, scale): the true state is scale * (mem, cnt).
// A step reads k rows (before the write, as the reference does), then applies the fade lazily: scale <- scale*lam
// and the k written rows get ww * v / scale.  So a step touches 2k rows instead of decaying all M rows.  When
// scale falls below 2^-60 the head's state is renormalised once (one pass, amortised over >= 1/log2(1/lam)*60
// steps).  Fade 0 is special: the state after a write is exactly that write, so the rows written at the previous
// step (last_w) are cleared instead.  One CTA per (stream, head); thread c owns value column c (thread 0 also the
// slot counts and the per-head words), so after one barrier (everyone has read scale and last_w) no two threads
// touch the same word.
#include "kernels.cuh"

namespace sdm {

__global__ void rt_decode_kernel(DecodeArgs a) {
  const int sh = blockIdx.x;
  const int hh = sh % a.h;
  const int s = sh / a.h;
  const int M = a.M, dh = a.dh, k = a.k;
  float* mem = a.mem + (int64_t)sh * M * dh;
  float* cnt = a.cnt + (int64_t)sh * M;
  int32_t* lw = a.last_w + (int64_t)sh * k;
  const int32_t* sir = a.sir + (int64_t)sh * k;
  const int32_t* siw = a.siw + (int64_t)sh * k;
  const float* wr = a.wr + (int64_t)sh * k;
  const float* ww = a.ww + (int64_t)sh * k;
  const float lam = a.decay[hh];
  // every thread reads the shared per-head words (scale, last written rows) before thread 0 rewrites them
  const float sc = a.scale[sh];
  int prev[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) prev[j] = j < k ? lw[j] : -1;
  const bool reset = a.reset && a.reset[s];
  __syncthreads();
  const int c = threadIdx.x;
  if (c >= dh) return;
  const bool own_cnt = (c == 0);
  if (reset) {
    for (int r = 0; r < M; ++r) mem[(int64_t)r * dh + c] = 0.f;
    if (own_cnt)
      for (int r = 0; r < M; ++r) cnt[r] = 0.f;
  }
  const float scr = reset ? 1.f : sc;
  // read k rows before the write: all k loads issued before the first use
  float rv[32], rc[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    if (i < k) {
      const int r = min(max(sir[i], 0), M - 1);  // slot ids are clamped into the state (see rt_scan.cu)
      rv[i] = mem[(int64_t)r * dh + c];
      rc[i] = own_cnt ? cnt[r] : 0.f;
    }
  }
  float acc = 0.f, accd = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    if (i < k) {
      acc = fmaf(wr[i], rv[i], acc);
      accd = fmaf(wr[i], rc[i], accd);
    }
  }
  a.num[(int64_t)sh * dh + c] = acc * scr;
  if (own_cnt) a.den[sh] = accd * scr;
  // write: state <- lam * state + sum_j ww_j (e_{siw_j} v^T, e_{siw_j})
  const float* v = a.V + (int64_t)s * a.ldv + (int64_t)hh * dh;
  float ns;
  if (lam == 0.f) {
    if (!reset) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int r = prev[j];
        if (r >= 0 && r < M) {
          mem[(int64_t)r * dh + c] = 0.f;
          if (own_cnt) cnt[r] = 0.f;
        }
      }
    }
    ns = 1.f;
  } else {
    ns = scr * lam;
    if (ns < 8.673617e-19f) {  // 2^-60: fold the scale into the state
      for (int r = 0; r < M; ++r) mem[(int64_t)r * dh + c] *= ns;
      if (own_cnt)
        for (int r = 0; r < M; ++r) cnt[r] *= ns;
      ns = 1.f;
    }
  }
  const float vc = v[c];
  // the k written rows are distinct (a top-k): load them all, then store them all.  With fade 0 every row that
  // is not cleared above is already zero, so the written value is the write alone.
  const bool keep_old = lam != 0.f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (j < k) {
      const int r = min(max(siw[j], 0), M - 1);
      rv[j] = keep_old ? mem[(int64_t)r * dh + c] : 0.f;
      rc[j] = (keep_old && own_cnt) ? cnt[r] : 0.f;
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (j < k) {
      const int r = min(max(siw[j], 0), M - 1);
      const float f = __fdiv_rn(ww[j], ns);
      mem[(int64_t)r * dh + c] = fmaf(f, vc, rv[j]);
      if (own_cnt) cnt[r] = rc[j] + f;
    }
  }
  if (own_cnt) {
    a.scale[sh] = ns;
    for (int j = 0; j < k; ++j) lw[j] = min(max(siw[j], 0), M - 1);
  }
}

cudaError_t launch_rt_decode(const DecodeArgs& a, cudaStream_t st) {
  if (a.S == 0) return cudaSuccess;
  const int threads = ((a.dh + 31) / 32) * 32;  // one thread per value column (dh <= 1024)
  LaunchScope scope_("rt_decode", st);
  rt_decode_kernel<<<(unsigned)((int64_t)a.S * a.h), threads, 0, st>>>(a);
  return cudaGetLastError();
}

// ----------------------------------------------------------------------------------------------- tied head
// Cross-entropy of one logits row (logsumexp - target logit), summed into a float64 total (ce_chunked's
// F.cross_entropy(..., reduction="sum"), track4_sdmllm24_fused_ce.py:76-77).  One block per row.
__global__ void ce_rows_kernel(const float* __restrict__ lg, int64_t rows, int V, const int32_t* __restrict__ tgt,
                               double* loss_sum) {
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
  ce_combine_kernel<<<(unsigned)ceil_div(rows, 8), 256, 0, st>>>(part, tgt_logit, targets, rows, tiles_n, loss_sum);
  return cudaGetLastError();
}

cudaError_t launch_argmax_combine(const float2* part, int64_t rows, int tiles_n, int32_t* ids, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  LaunchScope scope_("argmax_combine", st);
  argmax_combine_kernel<<<(unsigned)ceil_div(rows, 8), 256, 0, st>>>(part, rows, tiles_n, ids);
  return cudaGetLastError();
}

cudaError_t launch_ce_rows(const float* logits, int64_t rows, int V, const int32_t* targets, double* loss_sum,
                           cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  LaunchScope scope_("ce_rows", st);
  ce_rows_kernel<<<(unsigned)rows, 256, 0, st>>>(logits, rows, V, targets, loss_sum);
  return cudaGetLastError();
}
cudaError_t launch_argmax_rows(const float* logits, int64_t rows, int V, int32_t* ids, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  LaunchScope scope_("argmax_rows", st);
  argmax_rows_kernel<<<(unsigned)rows, 256, 0, st>>>(logits, rows, V, ids);
  return cudaGetLastError();
}

}  // namespace sdm
