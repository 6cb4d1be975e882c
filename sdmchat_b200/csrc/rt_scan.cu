// The run-time memory's write-then-read over a whole window (RunTimeSdm.forward's chunk loop,
// track4_onesdm_models.py:215-241 and :255-272), with the per-head state resident in shared memory.
//
// One CTA owns one (batch row b, head hh, slice of SCAN_CW value columns) for the WHOLE window: its slice of
// mem (M x SCAN_CW float32) and the slot counts cnt (M) live in shared memory from the first token to the last,
// so the state never travels through HBM (the reference's chunked form re-reads and re-writes it every chunk).
// Columns are independent in the recurrence, so slices of one head never communicate.
//
// Schedule: micro-steps of up to 16 tokens.  Within a step every token reads in parallel (one warp per token): the
// exact state at the step start, faded lam^(t-t0), plus the writes of earlier tokens of the same step to the slots
// it reads, found through a per-step slot list (with 16 tokens x k writes over M slots such collisions are rare).
// Then the step's writes go straight into the state, one job per distinct written slot, jobs dealt round-robin to
// the warps; a job walks its slot's list (every write to that slot in this step, newest first).  That is the
// reference's math (chunked form = token recurrence, :728-755) with a step of 16:
//   read   num[t] = sum_i wr[t,i] * ( lam^(t-t0) * mem[sir[t,i]] + sum_{t0<=s<t, siw[s,j]=sir[t,i]}
//                                                                      lam^(t-1-s) * ww[s,j] * v[s] )
//   write  mem <- lam^U * mem + sum_{s, j} lam^(t0+U-1-s) * ww[s,j] * e_{siw[s,j]} v[s]^T
// The fade is applied lazily: the state is held as sigma * P and a step multiplies sigma by lam^U instead of
// touching every row; writes add their term / sigma.  P is renormalised (one pass) when sigma would fall below
// 2^-40.  Fade 1 keeps sigma = 1; fade 0 (and fades below 2^-100) keep only the last token's writes.  A BOS reset
// (:229-233) starts a new step and empties the state.
//
// Lanes work in four groups of eight: a group covers one 32-column row with one 16-byte access per lane, so a
// warp touches four rows per shared-memory instruction (each quarter-warp phase reads one 128-byte row: no bank
// conflicts).  A token's k reads are taken four at a time and the four partial sums combined with two shuffles;
// write jobs are taken four at a time, one per group.
//
// Warps 0-15 ("workers") read and write, synchronising among themselves with a named barrier between the two
// phases; warp 16 ("builder") builds the NEXT step's slot lists and job list meanwhile (double-buffered) and
// meets the workers only at the step boundary.  Chunk inputs (slot ids, weights, values of 128 tokens) are
// prefetched into registers one chunk ahead.  No atomics touch float data and every sum runs in a fixed order, so
// results are bit-reproducible.
#include "kernels.cuh"

namespace sdm {

constexpr int SCAN_CW = 32;                            // value columns per CTA
constexpr int SCAN_WORKERS = 16;                       // warps that read and write
constexpr int SCAN_THREADS = (SCAN_WORKERS + 1) * 32;  // + the list-builder warp
constexpr int SCAN_U = 16;                             // tokens per micro-step (max)
constexpr int SCAN_MAX_ENTRIES = 2048;                 // L * k of one prefetched chunk
constexpr int SCAN_MAX_L = 128;
constexpr int SCAN_MAX_K = 32;
constexpr int SCAN_EB = SCAN_U * SCAN_MAX_K;           // entries (and jobs) per list buffer
constexpr int PF_E = SCAN_MAX_ENTRIES / (SCAN_WORKERS * 32);
constexpr int PF_V = SCAN_MAX_L * SCAN_CW / (SCAN_WORKERS * 32);

struct ScanSmem {
  size_t P, Pc, siw, ww, sir, wr, Vs, rst, head, nxt, ent_s, ent_w, jobs, lastr, total;
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
  s.rst = take((size_t)L * 4);
  s.head = take((size_t)2 * M * 4);
  s.nxt = take((size_t)2 * SCAN_EB * 4);
  s.ent_s = take((size_t)2 * SCAN_EB * 4);
  s.ent_w = take((size_t)2 * SCAN_EB * 4);
  s.jobs = take((size_t)2 * (SCAN_EB + 1) * 4);
  s.lastr = take((size_t)2 * SCAN_MAX_K * 4);
  s.total = o;
  return s;
}

static int scan_chunk_len(int k) {
  int L = SCAN_MAX_ENTRIES / k;
  return L > SCAN_MAX_L ? SCAN_MAX_L : L;
}

__device__ __forceinline__ void workers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(SCAN_WORKERS * 32) : "memory"); }

__device__ __forceinline__ void fma4(float4& acc, float w, const float4& v) {
  acc.x = fmaf(w, v.x, acc.x);
  acc.y = fmaf(w, v.y, acc.y);
  acc.z = fmaf(w, v.z, acc.z);
  acc.w = fmaf(w, v.w, acc.w);
}

// Inputs of one chunk held in registers between their load and their store to shared memory (worker warps).
struct Prefetch {
  int siw[PF_E], sir[PF_E];
  float ww[PF_E], wr[PF_E], v[PF_V];
  int rst;
};

__device__ __forceinline__ void prefetch_load(Prefetch& pf, const ScanArgs& a, int b, int hh, int cs, int c0,
                                              int Lc) {
  const int tid = threadIdx.x, k = a.k, nk = Lc * k;
  const int64_t base = (((int64_t)b * a.h + hh) * a.T + c0) * k;
#pragma unroll
  for (int q = 0; q < PF_E; ++q) {
    const int e = tid + q * SCAN_WORKERS * 32;
    if (e < nk) {
      pf.siw[q] = a.siw[base + e];
      pf.ww[q] = a.ww[base + e];
      pf.sir[q] = a.sir[base + e];
      pf.wr[q] = a.wr[base + e];
    }
  }
#pragma unroll
  for (int q = 0; q < PF_V; ++q) {
    const int i = tid + q * SCAN_WORKERS * 32;
    const int s = i / SCAN_CW, c = i % SCAN_CW, gc = cs * SCAN_CW + c;
    pf.v[q] = (s < Lc && gc < a.dh) ? a.V[((int64_t)b * a.T + c0 + s) * a.ldv + (int64_t)hh * a.dh + gc] : 0.f;
  }
  pf.rst = (a.reset && tid < Lc) ? (int)a.reset[(int64_t)b * a.T + c0 + tid] : 0;
}

__device__ __forceinline__ void prefetch_store(const Prefetch& pf, int M, int k, int Lc, int* siw_s, float* ww_s,
                                               int* sir_s, float* wr_s, float* Vs, int* rst_s) {
  const int tid = threadIdx.x, nk = Lc * k;
#pragma unroll
  for (int q = 0; q < PF_E; ++q) {
    const int e = tid + q * SCAN_WORKERS * 32;
    if (e < nk) {
      // slot ids outside [0, M) (never produced by the address kernel) are clamped so no access leaves the state
      siw_s[e] = min(max(pf.siw[q], 0), M - 1);
      ww_s[e] = pf.ww[q];
      sir_s[e] = min(max(pf.sir[q], 0), M - 1);
      wr_s[e] = pf.wr[q];
    }
  }
#pragma unroll
  for (int q = 0; q < PF_V; ++q) {
    const int i = tid + q * SCAN_WORKERS * 32;
    if (i < Lc * SCAN_CW) Vs[i] = pf.v[q];
  }
  if (tid < Lc) rst_s[tid] = pf.rst;
}

// Length of the micro-step starting at chunk position t0: at most ustep tokens, within the chunk, and cut before
// any BOS reset after t0 (a reset always starts a step).
__device__ __forceinline__ int step_len(int t0, int Lc, int ustep, const int* rst_s, bool has_reset) {
  int ue = min(ustep, Lc - t0);
  if (has_reset)
    for (int q = 1; q < ue; ++q)
      if (rst_s[t0 + q]) return q;
  return ue;
}

// The builder warp's lists for the step [t0, t0 + ue).  Entry e = q*k + j is write j of token t0 + q.
// head[r] = newest entry writing slot r (-1 if none), nxt[e] = next older entry of the same slot, ent_s / ent_w =
// chunk position and weight of e, jobs[1..] = the distinct written slots in first-write order, jobs[0] = count.
// Tokens are inserted 32/k at a time; writes of one group to the same slot are ordered with __match_any_sync.
template <int K>
__device__ __forceinline__ void build_lists(int t0, int ue, int k_rt, int M, const int* siw_s, const float* ww_s,
                                            int* head, int* nxt, int* ent_s, float* ent_w, int* jobs) {
  const int k = K > 0 ? K : k_rt;
  const int lane = threadIdx.x & 31;
  const unsigned FULL = 0xffffffffu;
  const int G = 32 / k;  // tokens per group
  const int ql = lane / k, jl = lane % k;
  int njobs = 0;
  for (int g0 = 0; g0 < ue; g0 += G) {
    const int q = g0 + ql;
    const bool valid = lane < G * k && q < ue;
    const int e = g0 * k + lane;
    const int s = t0 + q;
    const int r = valid ? siw_s[s * k + jl] : M + lane;  // invalid lanes match nothing
    const unsigned peers = __match_any_sync(FULL, r);
    const unsigned lower = peers & ((1u << lane) - 1u);
    const unsigned higher = peers & ~((2u << lane) - 1u);
    const int old_head = valid ? head[r] : -1;
    if (valid) {
      nxt[e] = lower ? g0 * k + (31 - __clz(lower)) : old_head;
      ent_s[e] = s;
      ent_w[e] = ww_s[s * k + jl];
    }
    __syncwarp();
    if (valid && higher == 0) head[r] = e;
    const bool newjob = valid && old_head < 0 && lower == 0;
    const unsigned jm = __ballot_sync(FULL, newjob);
    if (newjob) jobs[1 + njobs + __popc(jm & ((1u << lane) - 1u))] = r;
    njobs += __popc(jm);
    __syncwarp();
  }
  if (lane == 0) jobs[0] = njobs;
  __syncwarp();
}

template <int K>
__global__ void __launch_bounds__(SCAN_THREADS, 1) rt_scan_kernel(ScanArgs a, int L, int n_slices) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ float lampow[SCAN_U + 2];
  const int M = a.M, dh = a.dh, T = a.T, h = a.h;
  const int k = K > 0 ? K : a.k;
  constexpr int KR = K > 0 ? K : SCAN_MAX_K;  // unroll bound of the per-read loops
  const ScanSmem lay = scan_layout(M, L, k);
  float* P = reinterpret_cast<float*>(smem + lay.P);
  float4* P4 = reinterpret_cast<float4*>(smem + lay.P);
  float* Pc = reinterpret_cast<float*>(smem + lay.Pc);
  int* siw_s = reinterpret_cast<int*>(smem + lay.siw);
  float* ww_s = reinterpret_cast<float*>(smem + lay.ww);
  int* sir_s = reinterpret_cast<int*>(smem + lay.sir);
  float* wr_s = reinterpret_cast<float*>(smem + lay.wr);
  float* Vs = reinterpret_cast<float*>(smem + lay.Vs);
  const float4* Vs4 = reinterpret_cast<const float4*>(smem + lay.Vs);
  int* rst_s = reinterpret_cast<int*>(smem + lay.rst);
  int* head_b = reinterpret_cast<int*>(smem + lay.head);
  int* nxt_b = reinterpret_cast<int*>(smem + lay.nxt);
  int* ents_b = reinterpret_cast<int*>(smem + lay.ent_s);
  float* entw_b = reinterpret_cast<float*>(smem + lay.ent_w);
  int* jobs_b = reinterpret_cast<int*>(smem + lay.jobs);
  int* lastr_b = reinterpret_cast<int*>(smem + lay.lastr);

  const int cs = blockIdx.x % n_slices;
  const int bh = blockIdx.x / n_slices;
  const int hh = bh % h;
  const int b = bh / h;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = lane >> 3, c4 = lane & 7;  // lane group (row) and its 4-column quad
  const bool builder = warp == SCAN_WORKERS;
  const int ncols = min(SCAN_CW, dh - cs * SCAN_CW);  // valid columns of this slice
  const float lam = a.decay[hh];
  const bool has_reset = a.reset != nullptr;
  const unsigned FULL = 0xffffffffu;
  // fade mode: 0 = only the last token's writes survive (lam = 0 or below 2^-100), 1 = no fade, 2 = lazy scale
  const int mode = (lam < 7.8886e-31f) ? 0 : (lam == 1.f ? 1 : 2);
  int ustep = SCAN_U;
  if (mode == 2 && lam < 0.0131f) ustep = max(1, min(SCAN_U, (int)floorf(100.f / -log2f(lam))));  // lam^U >= 2^-100

  for (int i = tid; i < M * (SCAN_CW / 4); i += SCAN_THREADS) P4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int i = tid; i < M; i += SCAN_THREADS) {
    Pc[i] = 0.f;
    head_b[i] = -1;
    head_b[M + i] = -1;
  }
  if (tid <= SCAN_U) lampow[tid] = mode == 0 ? (tid == 0 ? 1.f : 0.f) : powf(lam, (float)tid);
  if (tid < 2 * SCAN_MAX_K) lastr_b[tid] = -1;
  float sigma = 1.f;  // state = sigma * P (mode 2)
  Prefetch pf;
  if (!builder) {
    const int Lc0 = min(L, T);
    prefetch_load(pf, a, b, hh, cs, 0, Lc0);
    prefetch_store(pf, M, k, Lc0, siw_s, ww_s, sir_s, wr_s, Vs, rst_s);
  }
  __syncthreads();
  int buf = 0;   // list buffer of the current step
  int lbuf = 0;  // survivor-row buffer (fade 0)

  for (int c0 = 0; c0 < T; c0 += L) {
    const int Lc = min(L, T - c0);
    const int c0n = c0 + L;
    const int Lcn = c0n < T ? min(L, T - c0n) : 0;
    if (!builder && Lcn > 0) prefetch_load(pf, a, b, hh, cs, c0n, Lcn);  // lands while this chunk computes
    if (builder)
      build_lists<K>(0, step_len(0, Lc, ustep, rst_s, has_reset), k, M, siw_s, ww_s, head_b + buf * M,
                     nxt_b + buf * SCAN_EB, ents_b + buf * SCAN_EB, entw_b + buf * SCAN_EB,
                     jobs_b + buf * (SCAN_EB + 1));
    __syncthreads();

    for (int t0 = 0; t0 < Lc;) {
      const int ue = step_len(t0, Lc, ustep, rst_s, has_reset);
      const int t1 = t0 + ue;
      if (builder) {
        // the next step's lists, into the other buffer (its heads were cleared by the previous step's writes)
        if (t1 < Lc) {
          const int nb = buf ^ 1;
          build_lists<K>(t1, step_len(t1, Lc, ustep, rst_s, has_reset), k, M, siw_s, ww_s, head_b + nb * M,
                         nxt_b + nb * SCAN_EB, ents_b + nb * SCAN_EB, entw_b + nb * SCAN_EB,
                         jobs_b + nb * (SCAN_EB + 1));
        }
      } else {
        int* head = head_b + buf * M;
        const int* nxt = nxt_b + buf * SCAN_EB;
        const int* ent_s = ents_b + buf * SCAN_EB;
        const float* ent_w = entw_b + buf * SCAN_EB;
        const int* jobs = jobs_b + buf * (SCAN_EB + 1);
        // a BOS empties the memory before its token reads; a tiny scale is folded into the state
        const bool clear = has_reset && rst_s[t0] != 0;
        const bool renorm = !clear && mode == 2 && sigma * lampow[ue] < 9.094947e-13f;  // 2^-40
        if (clear || renorm) {
          const float f = clear ? 0.f : sigma;
          for (int i = tid; i < M * (SCAN_CW / 4); i += SCAN_WORKERS * 32) {
            float4 v = P4[i];
            P4[i] = make_float4(v.x * f, v.y * f, v.z * f, v.w * f);
          }
          for (int i = tid; i < M; i += SCAN_WORKERS * 32) Pc[i] *= f;
          if (clear && tid < SCAN_MAX_K) lastr_b[lbuf * SCAN_MAX_K + tid] = -1;
          sigma = 1.f;
          workers_sync();
        }

        // reads: worker warp w takes token t0 + w; group g handles reads g, g+4, ...
        if (warp < ue) {
          const int tau = t0 + warp;
          const float fade = (mode == 2 ? sigma : 1.f) * lampow[warp];
          int ri = 0, hd = -1;
          float wi = 0.f, pdi = 0.f;
          if (lane < k) {
            ri = sir_s[tau * k + lane];
            wi = wr_s[tau * k + lane];
            pdi = Pc[ri];
            hd = head[ri];
          }
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int q = 0; q < (KR + 3) / 4; ++q) {
            const int ii = 4 * q + grp;
            const int r = __shfl_sync(FULL, ri, ii & 31);
            const float w = __shfl_sync(FULL, wi, ii & 31);
            if (K > 0 ? (ii < K) : (ii < k)) fma4(acc, w, P4[r * (SCAN_CW / 4) + c4]);
          }
#pragma unroll
          for (int o = 8; o < 32; o <<= 1) {
            acc.x += __shfl_xor_sync(FULL, acc.x, o);
            acc.y += __shfl_xor_sync(FULL, acc.y, o);
            acc.z += __shfl_xor_sync(FULL, acc.z, o);
            acc.w += __shfl_xor_sync(FULL, acc.w, o);
          }
          const float dcar = warp_sum(wi * pdi);
          float4 iv = make_float4(0.f, 0.f, 0.f, 0.f);
          float idn = 0.f;
          unsigned mask = __ballot_sync(FULL, hd >= 0);
          while (mask) {
            const int i = __ffs(mask) - 1;
            mask &= mask - 1u;
            const float w = __shfl_sync(FULL, wi, i);
            for (int e = __shfl_sync(FULL, hd, i); e >= 0; e = nxt[e]) {
              const int s = ent_s[e];
              if (s >= tau) continue;
              const float coef = w * ent_w[e] * lampow[tau - 1 - s];
              fma4(iv, coef, Vs4[s * (SCAN_CW / 4) + c4]);
              idn += coef;
            }
          }
          const int64_t tok = (int64_t)b * T + c0 + tau;
          if (grp == 0) {
            float* dst = a.num + (tok * h + hh) * dh + cs * SCAN_CW + 4 * c4;
            const float o0 = fmaf(fade, acc.x, iv.x), o1 = fmaf(fade, acc.y, iv.y);
            const float o2 = fmaf(fade, acc.z, iv.z), o3 = fmaf(fade, acc.w, iv.w);
            if (4 * c4 + 3 < ncols && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
              *reinterpret_cast<float4*>(dst) = make_float4(o0, o1, o2, o3);
            } else {
              if (4 * c4 + 0 < ncols) dst[0] = o0;
              if (4 * c4 + 1 < ncols) dst[1] = o1;
              if (4 * c4 + 2 < ncols) dst[2] = o2;
              if (4 * c4 + 3 < ncols) dst[3] = o3;
            }
          }
          if (cs == 0 && lane == 0) a.den[tok * h + hh] = fmaf(fade, dcar, idn);
        }
        workers_sync();

        // writes
        const int njobs = jobs[0];
        if (mode != 0) {
          const float inv = mode == 2 ? 1.f / (sigma * lampow[ue]) : 1.f;
          for (int jb = 4 * warp; jb < njobs; jb += 4 * SCAN_WORKERS) {
            const int j = jb + grp;
            const bool valid = j < njobs;
            const int r = valid ? jobs[1 + j] : 0;
            int e = valid ? head[r] : -1;
            float4 p = make_float4(0.f, 0.f, 0.f, 0.f);
            float pc = 0.f;
            if (valid) {
              p = P4[r * (SCAN_CW / 4) + c4];
              pc = Pc[r];
            }
            while (e >= 0) {
              const int se = ent_s[e];
              const float f = ent_w[e] * lampow[t1 - 1 - se] * inv;
              fma4(p, f, Vs4[se * (SCAN_CW / 4) + c4]);
              pc += f;
              e = nxt[e];
            }
            __syncwarp();
            if (valid) {
              P4[r * (SCAN_CW / 4) + c4] = p;
              if (c4 == 0) {
                Pc[r] = pc;
                head[r] = -1;
              }
            }
          }
          if (mode == 2) sigma *= lampow[ue];
        } else {
          // fade 0: the state becomes the step's last token's writes alone.  Row jj: set new row jj and clear
          // old survivor row jj unless it is among the new rows (the two sets of rows touched are disjoint).
          const int sl = t1 - 1;
          const int* lold = lastr_b + lbuf * SCAN_MAX_K;
          int* lnew = lastr_b + (lbuf ^ 1) * SCAN_MAX_K;
          const int rn_l = lane < k ? siw_s[sl * k + lane] : -2;
          for (int j0 = 4 * warp; j0 < k; j0 += 4 * SCAN_WORKERS) {
            const int jj = j0 + grp;
            const bool valid = jj < k;
            const int rn = valid ? siw_s[sl * k + jj] : 0;
            const int ro = valid ? lold[jj] : -1;
            bool old_in_new = false;
#pragma unroll
            for (int l = 0; l < SCAN_MAX_K; ++l) {
              const int rl = __shfl_sync(FULL, rn_l, l);
              old_in_new |= (rl == ro);
            }
            if (valid) {
              const float wn = ww_s[sl * k + jj];
              const float4 v = Vs4[sl * (SCAN_CW / 4) + c4];
              P4[rn * (SCAN_CW / 4) + c4] = make_float4(wn * v.x, wn * v.y, wn * v.z, wn * v.w);
              if (c4 == 0) {
                Pc[rn] = wn;
                lnew[jj] = rn;
              }
              if (ro >= 0 && !old_in_new) {
                P4[ro * (SCAN_CW / 4) + c4] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (c4 == 0) Pc[ro] = 0.f;
              }
            }
          }
          for (int jb = warp; jb < njobs; jb += SCAN_WORKERS)
            if (lane == 0) head[jobs[1 + jb]] = -1;
          lbuf ^= 1;
        }
      }
      buf ^= 1;
      t0 = t1;
      __syncthreads();
    }
    // the next chunk's inputs
    if (Lcn > 0) {
      if (!builder) prefetch_store(pf, M, k, Lcn, siw_s, ww_s, sir_s, wr_s, Vs, rst_s);
      __syncthreads();
    }
  }
  // the final state, unscaled
  if (!builder) {
    const float fs = mode == 2 ? sigma : 1.f;
    if (a.mem_out) {
      float* mo = a.mem_out + ((int64_t)b * h + hh) * (int64_t)M * dh;
      for (int i = tid; i < M * SCAN_CW; i += SCAN_WORKERS * 32) {
        const int r = i / SCAN_CW, c = i % SCAN_CW, gc = cs * SCAN_CW + c;
        if (gc < dh) mo[(int64_t)r * dh + gc] = P[i] * fs;
      }
    }
    if (a.cnt_out && cs == 0) {
      float* co = a.cnt_out + ((int64_t)b * h + hh) * (int64_t)M;
      for (int r = tid; r < M; r += SCAN_WORKERS * 32) co[r] = Pc[r] * fs;
    }
  }
}

bool rt_scan_supported(int M, int dh, int k) {
  if (M < 1 || dh < 1 || k < 1 || k > SCAN_MAX_K) return false;
  return scan_layout(M, scan_chunk_len(k), k).total <= 227 * 1024;
}

template <int K>
static cudaError_t launch_scan_k(const ScanArgs& a, int L, size_t smem, int n_slices, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(rt_scan_kernel<K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int64_t grid = (int64_t)a.B * a.h * n_slices;
  LaunchScope scope_("rt_scan", st);
  rt_scan_kernel<K><<<(unsigned)grid, SCAN_THREADS, smem, st>>>(a, L, n_slices);
  return cudaGetLastError();
}

cudaError_t launch_rt_scan(const ScanArgs& a, cudaStream_t st) {
  if (a.B == 0 || a.T == 0) return cudaSuccess;
  const int L = scan_chunk_len(a.k);
  const size_t smem = scan_layout(a.M, L, a.k).total;
  const int n_slices = (a.dh + SCAN_CW - 1) / SCAN_CW;
  switch (a.k) {
    case 16: return launch_scan_k<16>(a, L, smem, n_slices, st);
    case 4: return launch_scan_k<4>(a, L, smem, n_slices, st);
    default: return launch_scan_k<0>(a, L, smem, n_slices, st);
  }
}

}  // namespace sdm
