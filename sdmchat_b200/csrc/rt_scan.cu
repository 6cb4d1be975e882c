// The run-time memory's write-then-read over a whole window (RunTimeSdm._chunk over every chunk,
// track4_onesdm_models.py:215-241 and the loop :255-272), with the per-head state resident in shared memory.
//
// One CTA owns one (batch row b, head hh, slice of SCAN_CW value columns) for the WHOLE window: its slice of
// mem (M x SCAN_CW float32) and the slot counts cnt (M) live in shared memory from the first token to the last,
// so the state never travels through HBM (the reference's chunked form re-reads and re-writes it every chunk).
// Columns are independent in the recurrence, so slices of one head never communicate.
//
// Per chunk of L tokens (the reference's math, sparse):
//   read   num[t] = sum_i wr[t,i] * ( lam^(t-c0) * mem[sir[t,i]]  +  sum_{s<t in chunk, siw[s,j]=sir[t,i]}
//                                                                      lam^(t-1-s) * ww[s,j] * v[s] )
//   write  mem[r] <- lam^L * mem[r] + sum_{s, j: siw[s,j]=r} lam^(L-1-s) * ww[s,j] * v[s]
// with cnt the same recurrence on a value of 1.  The chunk's L*k writes are bucketed by slot (a counting sort in
// shared memory, each bucket in (s, j) order) so a read finds the earlier in-chunk writes to its slot, and the
// write phase walks every slot once (its decay plus its bucket).  Reads of the whole chunk run in parallel (one
// warp per token, one lane per column), then the writes (one warp per slot); no atomics touch float data, so
// results are bit-reproducible.  BOS resets (:229-233) mask by segment number exactly as the reference does.
#include "kernels.cuh"

namespace sdm {

constexpr int SCAN_CW = 32;        // value columns per CTA
constexpr int SCAN_THREADS = 512;  // 16 warps
constexpr int SCAN_MAX_ENTRIES = 2048;  // L * k per chunk

struct ScanSmem {
  size_t P, Pc, siw, ww, sir, wr, Vs, bstart, bcount, entries, lampow, seg, total;
};

__host__ __device__ inline ScanSmem scan_layout(int M, int L, int k) {
  ScanSmem s;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    size_t r = o;
    o += (bytes + 15) & ~(size_t)15;
    return r;
  };
  s.P = take((size_t)M * SCAN_CW * 4);
  s.Pc = take((size_t)M * 4);
  s.siw = take((size_t)L * k * 4);
  s.ww = take((size_t)L * k * 4);
  s.sir = take((size_t)L * k * 4);
  s.wr = take((size_t)L * k * 4);
  s.Vs = take((size_t)L * SCAN_CW * 4);
  s.bstart = take((size_t)(M + 1) * 4);
  s.bcount = take((size_t)M * 4);
  s.entries = take((size_t)L * k * 8);
  s.lampow = take((size_t)(L + 1) * 4);
  s.seg = take((size_t)L * 4);
  s.total = o;
  return s;
}

static int scan_chunk_len(int k) {
  int L = SCAN_MAX_ENTRIES / k;
  return L > 128 ? 128 : L;
}

// Exclusive prefix sum of cnt[0..M) into start[0..M] (start[M] = total) by the whole block.
__device__ void block_exclusive_scan(const int* cnt, int* start, int M, int* warp_tot) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (M + SCAN_THREADS - 1) / SCAN_THREADS;
  const int lo = tid * per;
  int local = 0;
  for (int q = 0; q < per; ++q)
    if (lo + q < M) local += cnt[lo + q];
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int v = lane < SCAN_THREADS / 32 ? warp_tot[lane] : 0;
    int inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int u = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += u;
    }
    if (lane < SCAN_THREADS / 32) warp_tot[lane] = inc - v;  // exclusive warp offsets
  }
  __syncthreads();
  int run = warp_tot[warp] + incl - local;
  for (int q = 0; q < per; ++q) {
    if (lo + q < M) {
      start[lo + q] = run;
      run += cnt[lo + q];
    }
  }
  if (tid == SCAN_THREADS - 1) start[M] = run;
  __syncthreads();
}

__global__ void __launch_bounds__(SCAN_THREADS, 1) rt_scan_kernel(ScanArgs a, int L, int n_slices) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ int warp_tot[SCAN_THREADS / 32];
  const int M = a.M, k = a.k, dh = a.dh, T = a.T, h = a.h;
  const ScanSmem lay = scan_layout(M, L, k);
  float* P = reinterpret_cast<float*>(smem + lay.P);
  float* Pc = reinterpret_cast<float*>(smem + lay.Pc);
  int* siw_s = reinterpret_cast<int*>(smem + lay.siw);
  float* ww_s = reinterpret_cast<float*>(smem + lay.ww);
  int* sir_s = reinterpret_cast<int*>(smem + lay.sir);
  float* wr_s = reinterpret_cast<float*>(smem + lay.wr);
  float* Vs = reinterpret_cast<float*>(smem + lay.Vs);
  int* bstart = reinterpret_cast<int*>(smem + lay.bstart);
  int* bcount = reinterpret_cast<int*>(smem + lay.bcount);
  int2* entries = reinterpret_cast<int2*>(smem + lay.entries);
  float* lampow = reinterpret_cast<float*>(smem + lay.lampow);
  int* seg_s = reinterpret_cast<int*>(smem + lay.seg);

  const int cs = blockIdx.x % n_slices;
  const int bh = blockIdx.x / n_slices;
  const int hh = bh % h;
  const int b = bh / h;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NW = SCAN_THREADS / 32;
  const int col = cs * SCAN_CW + lane;
  const bool col_ok = col < dh;
  const float lam = a.decay[hh];
  const bool has_reset = a.reset != nullptr;

  for (int i = tid; i < M * SCAN_CW; i += SCAN_THREADS) P[i] = 0.f;
  for (int i = tid; i < M; i += SCAN_THREADS) Pc[i] = 0.f;
  for (int e = tid; e <= L; e += SCAN_THREADS) lampow[e] = powf(lam, (float)e);  // powf(0, 0) = 1, as torch.pow
  int seg_prev = 0;  // segment number of the position just before the chunk (BOS count so far)
  __syncthreads();

  for (int c0 = 0; c0 < T; c0 += L) {
    const int Lc = min(L, T - c0);
    const int nk = Lc * k;
    const int64_t base = (((int64_t)b * h + hh) * T + c0) * k;
    for (int e = tid; e < nk; e += SCAN_THREADS) {
      // slot ids outside [0, M) (never produced by the address kernel) are clamped so no access leaves the state
      siw_s[e] = min(max(a.siw[base + e], 0), M - 1);
      ww_s[e] = a.ww[base + e];
      sir_s[e] = min(max(a.sir[base + e], 0), M - 1);
      wr_s[e] = a.wr[base + e];
    }
    for (int i = tid; i < Lc * SCAN_CW; i += SCAN_THREADS) {
      const int s = i / SCAN_CW, c = i % SCAN_CW, gc = cs * SCAN_CW + c;
      Vs[i] = gc < dh ? a.V[((int64_t)b * T + c0 + s) * a.ldv + (int64_t)hh * dh + gc] : 0.f;
    }
    if (has_reset && warp == 0) {
      int run = seg_prev;
      for (int p0 = 0; p0 < Lc; p0 += 32) {
        const int s = p0 + lane;
        const bool f = s < Lc && a.reset[(int64_t)b * T + c0 + s] != 0;
        const unsigned m = __ballot_sync(0xffffffffu, f);
        if (s < Lc) seg_s[s] = run + __popc(m & (0xffffffffu >> (31 - lane)));
        run += __popc(m);
      }
    }
    for (int r = tid; r < M; r += SCAN_THREADS) bcount[r] = 0;
    __syncthreads();
    // bucket the chunk's writes by slot
    for (int e = tid; e < nk; e += SCAN_THREADS) atomicAdd(&bcount[siw_s[e]], 1);
    __syncthreads();
    block_exclusive_scan(bcount, bstart, M, warp_tot);
    for (int r = tid; r < M; r += SCAN_THREADS) bcount[r] = 0;
    __syncthreads();
    for (int e = tid; e < nk; e += SCAN_THREADS) {
      const int slot = siw_s[e];
      const int pos = bstart[slot] + atomicAdd(&bcount[slot], 1);
      entries[pos].x = e;
    }
    __syncthreads();
    for (int r = tid; r < M; r += SCAN_THREADS) {
      const int lo = bstart[r], hi = bstart[r + 1];
      for (int p = lo + 1; p < hi; ++p) {  // insertion sort: (s, j) order
        const int key = entries[p].x;
        int q = p - 1;
        while (q >= lo && entries[q].x > key) {
          entries[q + 1].x = entries[q].x;
          --q;
        }
        entries[q + 1].x = key;
      }
      for (int p = lo; p < hi; ++p) {
        const int e = entries[p].x;
        entries[p] = make_int2(e / k, __float_as_int(ww_s[e]));
      }
    }
    __syncthreads();
    // read phase: warp per token, lane per column
    for (int tau = warp; tau < Lc; tau += NW) {
      const int seg_t = has_reset ? seg_s[tau] : 0;
      const float fade = (!has_reset || seg_t == seg_prev) ? lampow[tau] : 0.f;
      float acc = 0.f, accd = 0.f;
      for (int i = 0; i < k; ++i) {
        const int r = sir_s[tau * k + i];
        const float w = wr_s[tau * k + i];
        const float pv = P[r * SCAN_CW + lane];
        const float pd = Pc[r];
        float iv = 0.f, id = 0.f;
        const int hi = bstart[r + 1];
        for (int p = bstart[r]; p < hi; ++p) {
          const int2 en = entries[p];
          if (en.x >= tau) break;
          if (has_reset && seg_s[en.x] != seg_t) continue;
          const float coef = __int_as_float(en.y) * lampow[tau - 1 - en.x];
          iv = fmaf(coef, Vs[en.x * SCAN_CW + lane], iv);
          id += coef;
        }
        acc = fmaf(w, fmaf(fade, pv, iv), acc);
        accd = fmaf(w, fmaf(fade, pd, id), accd);
      }
      const int64_t tok = (int64_t)b * T + c0 + tau;
      if (col_ok) a.num[(tok * h + hh) * dh + col] = acc;
      if (cs == 0 && lane == 0) a.den[tok * h + hh] = accd;
    }
    __syncthreads();
    // write phase: warp per slot, lane per column
    const int seg_last = has_reset ? seg_s[Lc - 1] : 0;
    const float dec = (!has_reset || seg_last == seg_prev) ? lampow[Lc] : 0.f;
    for (int r = warp; r < M; r += NW) {
      float pv = P[r * SCAN_CW + lane] * dec;
      float pc = Pc[r] * dec;
      const int hi = bstart[r + 1];
      for (int p = bstart[r]; p < hi; ++p) {
        const int2 en = entries[p];
        if (has_reset && seg_s[en.x] != seg_last) continue;
        const float f = __int_as_float(en.y) * lampow[Lc - 1 - en.x];
        pv = fmaf(f, Vs[en.x * SCAN_CW + lane], pv);
        pc += f;
      }
      P[r * SCAN_CW + lane] = pv;
      if (lane == 0) Pc[r] = pc;
    }
    if (has_reset) seg_prev = seg_last;
    __syncthreads();
  }
  if (a.mem_out) {
    float* mo = a.mem_out + ((int64_t)b * h + hh) * (int64_t)M * dh;
    for (int i = tid; i < M * SCAN_CW; i += SCAN_THREADS) {
      const int r = i / SCAN_CW, c = i % SCAN_CW, gc = cs * SCAN_CW + c;
      if (gc < dh) mo[(int64_t)r * dh + gc] = P[i];
    }
  }
  if (a.cnt_out && cs == 0) {
    float* co = a.cnt_out + ((int64_t)b * h + hh) * (int64_t)M;
    for (int r = tid; r < M; r += SCAN_THREADS) co[r] = Pc[r];
  }
}

bool rt_scan_supported(int M, int dh, int k) {
  if (M < 1 || dh < 1 || k < 1 || k > 32) return false;
  return scan_layout(M, scan_chunk_len(k), k).total <= 227 * 1024;
}

cudaError_t launch_rt_scan(const ScanArgs& a, cudaStream_t st) {
  if (a.B == 0 || a.T == 0) return cudaSuccess;
  const int L = scan_chunk_len(a.k);
  const ScanSmem lay = scan_layout(a.M, L, a.k);
  cudaError_t e = cudaFuncSetAttribute(rt_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lay.total);
  if (e != cudaSuccess) return e;
  const int n_slices = (a.dh + SCAN_CW - 1) / SCAN_CW;
  const int64_t grid = (int64_t)a.B * a.h * n_slices;
  LaunchScope scope_("rt_scan", st);
  rt_scan_kernel<<<(unsigned)grid, SCAN_THREADS, lay.total, st>>>(a, L, n_slices);
  return cudaGetLastError();
}

}  // namespace sdm
