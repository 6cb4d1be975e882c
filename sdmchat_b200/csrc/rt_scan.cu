// The run-time memory's write-then-read over a whole window (RunTimeSdm.forward's chunk loop,
// track4_onesdm_models.py:215-241 and :255-272, equal to the token recurrence of forward_sequential, :285-299).
//
// Per token t of head hh (fade lam, k reads and k writes per token):
//   read   num[t] = sum_i wr[t,i] * mem_t[sir[t,i]]            den[t] = sum_i wr[t,i] * cnt_t[sir[t,i]]
//   write  mem_{t+1} = lam * mem_t + sum_j ww[t,j] e_{siw[t,j]} v[t]^T      (cnt likewise with 1 for v)
// and a BOS reset at t empties the memory before t's read (:229-233).  Over a chunk [c0, c0 + Lc) this unrolls to
//   num[t] = lam^(t-c0) sum_i wr[t,i] mem_c0[sir[t,i]]                                  (the state part)
//          + sum_{c0<=s<t} lam^(t-1-s) sum_{i,j: sir[t,i]=siw[s,j]} wr[t,i] ww[s,j] v[s]    (the intra part)
//   mem_{c0+Lc} = lam^Lc mem_c0 + sum_{s,j} lam^(c0+Lc-1-s) ww[s,j] e_{siw[s,j]} v[s]^T
// The intra part and the slot lists of the state update depend on the chunk's own selections only, so they are
// computed for every (row, head, chunk) at once by rt_lists_kernel; only the state part is sequential, and
// rt_scan_kernel carries the state through the chunks of one (row, head) with all of a chunk's reads (and then
// all of its writes) in parallel: two or three CTA barriers per 64 tokens.
//
// rt_lists_kernel, one CTA per (b, hh, chunk):
//   * groups the chunk's k * Lc write entries by slot, in token order within a slot (a bit per (slot, token) in
//     shared memory: an entry's rank in its run is the number of earlier tokens that wrote the slot), so the
//     order is deterministic;
//   * intra part: eight lanes per token (each owning dh/8 columns); each of the token's k reads walks its slot's
//     run (entries of earlier tokens of the chunk, at or after the token's last reset) and adds coef * v[s];
//     writes num and den;
//   * the chunk record for the state scan: the distinct written slots ("jobs", runs of kLongRun or more entries
//     first so the long runs of repeated tokens start together) with their entries
//     (source token and coefficient ww * lam^(Lc-1-s)), restricted to entries after the chunk's last reset, and
//     the chunk header {njobs, nent, rd_end, clear}: tokens before the first reset (rd_end) read the state, a
//     reset anywhere in the chunk clears it before the writes.
//   Fade 0 (and fades below 2^-100): only the previous token's writes are visible, so the intra part compares
//   token t's reads with token t-1's writes (t-1 may be the last token of the previous chunk) and the state scan
//   only materialises the final state (the last token's writes).
//
// rt_scan_kernel, one CTA per (b, hh, slice of CW value columns): the slice of mem (M x CW float32) and
// cnt (M) stay in shared memory for the whole window.  Chunk inputs (record, read selections, value slice, the
// intra num/den) are copied with cp.async one chunk ahead into a second buffer; chunk headers are loaded two
// chunks ahead so every copy has its exact size.  32 warps per CTA.  A lane group of CW/4 lanes covers one CW-column
// row per 16-byte access (CW = 32: eight-lane groups; CW = 16, for batches too small to fill the SMs with 32-column
// slices: four-lane groups).  Per chunk: reads (each token's k reads in two halves, one lane group each, four read
// ids per 16-byte load) add the faded state part to num; then the jobs update the state (one lane group per slot:
// the sum of the slot's entries, then one read-modify-write).  The fade is lazy: the state is sigma * P, a chunk
// multiplies sigma by lam^Lc and writes add coef / sigma; when sigma would drop below 2^-40 the chunk instead scales
// P in one pass.  All sums run in a fixed order, the same for either slice width: results are bit-reproducible.
#include "kernels.cuh"
#include "tma.cuh"

namespace sdm {

constexpr int CH_MAX_E = 1024;  // write entries (tokens x k) of one chunk
constexpr int CH_MAX_L = 64;    // tokens of one chunk
constexpr int SCAN_MAX_K = 32;
constexpr int LIST_THREADS = 256;
constexpr int LIST_WARPS = LIST_THREADS / 32;
constexpr int LIST_MAX_DH = 256;
constexpr int SCAN_CW = 32;        // value columns per scan CTA
constexpr int SCAN_CW_SMALL = 16;  // ... when B x h x 32-column slices would fill at most half the SMs
constexpr int SCAN_WARPS = 32;
constexpr int SCAN_THREADS = SCAN_WARPS * 32;
constexpr float kTinyFade = 7.8886e-31f;  // 2^-100: fades below are treated as 0
constexpr float kRenorm = 9.094947e-13f;  // 2^-40

__host__ __device__ inline int chunk_len(int k) {
  const int L = CH_MAX_E / k;
  return L > CH_MAX_L ? CH_MAX_L : L;
}
__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~(size_t)15; }

// One chunk's record: jobs {slot, first entry | entry count << 16}, runs of kLongRun or more entries first, then
// entries {source token, coefficient bits} grouped by slot.  Headers {njobs, nent, rd_end, clear} are kept apart,
// one int4 per chunk.
constexpr int kLongRun = 4;
struct RecLayout {
  int E;
  size_t ents, bytes;
};
__host__ __device__ inline RecLayout rec_layout(int k) {
  RecLayout r;
  r.E = chunk_len(k) * k;
  r.ents = align16((size_t)r.E * 8);
  r.bytes = 2 * r.ents;
  return r;
}
__host__ __device__ inline size_t rec_region_bytes(int B, int T, int h, int k) {
  const int L = chunk_len(k);
  return (size_t)B * h * ((T + L - 1) / L) * rec_layout(k).bytes;
}

__device__ __forceinline__ int fade_mode(float lam) { return lam < kTinyFade ? 0 : (lam == 1.f ? 1 : 2); }

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// rows x w 4-byte elements from src (row stride `stride` elements) to dst (row pitch `pitch` elements), issued by
// threads [0, nt) as 16-byte copies when everything is 16-byte aligned, else as 4-byte copies.
__device__ __forceinline__ void copy_rows_async(void* dst, const void* src, int rows, int w, int pitch,
                                                int64_t stride, int tid, int nt) {
  const uint32_t* s = static_cast<const uint32_t*>(src);
  uint32_t* d = static_cast<uint32_t*>(dst);
  const bool vec = (reinterpret_cast<uintptr_t>(src) & 15) == 0 && (w & 3) == 0 && (pitch & 3) == 0 &&
                   (stride & 3) == 0;
  if (vec) {
    const int nv = w >> 2;
    for (int i = tid; i < rows * nv; i += nt) {
      const int r = i / nv, q = i - r * nv;
      cp_async16(d + (int64_t)r * pitch + 4 * q, s + r * stride + 4 * q);
    }
  } else {
    for (int i = tid; i < rows * w; i += nt) {
      const int r = i / w, q = i - r * w;
      cp_async4(d + (int64_t)r * pitch + q, s + r * stride + q);
    }
  }
}

// n contiguous 4-byte words, 16-byte copies when both ends are aligned.
__device__ __forceinline__ void copy_words_async(void* dst, const void* src, int n, int tid, int nt) {
  const uint32_t* s = static_cast<const uint32_t*>(src);
  uint32_t* d = static_cast<uint32_t*>(dst);
  int done = 0;
  if (((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d)) & 15) == 0) {
    const int nv = n >> 2;
    for (int i = tid; i < nv; i += nt) cp_async16(d + 4 * i, s + 4 * i);
    done = nv << 2;
  }
  for (int i = done + tid; i < n; i += nt) cp_async4(d + i, s + i);
}
// rows of cw words (w of them valid) with row stride `stride` words into rows of cw words.
__device__ __forceinline__ void copy_rows32_async(void* dst, const void* src, int rows, int w, int cw, int64_t stride,
                                                  int tid, int nt);

__device__ __forceinline__ void fma4(float4& acc, float w, const float4& v) {  // acc += w * v, as four fmaf
  const float2 ww = make_float2(w, w);
  const float2 lo = fma2(ww, make_float2(v.x, v.y), make_float2(acc.x, acc.y));
  const float2 hi = fma2(ww, make_float2(v.z, v.w), make_float2(acc.z, acc.w));
  acc = make_float4(lo.x, lo.y, hi.x, hi.y);
}

// Exclusive prefix sum of in(0) .. in(n-1) into out[0, n) by all LIST_THREADS threads (out must not be what in()
// reads); returns the total.  Ends with a barrier.  Thread t takes elements [t * per, (t + 1) * per); when that is
// four (n = 4 x LIST_THREADS, the usual 1,024 slots) it reads them as in4(t) = in(4t .. 4t + 3) and writes them
// with one 16-byte store, so a warp's accesses cover consecutive 16-byte words (no bank conflicts).
template <typename In, typename In4>
__device__ __forceinline__ int block_exclusive_scan(In in, In4 in4, int* out, int n, int* wtot) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (n + LIST_THREADS - 1) / LIST_THREADS;
  const bool v4 = n == 4 * LIST_THREADS && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  const int s0 = tid * per, s1 = min(n, s0 + per);
  int4 q = make_int4(0, 0, 0, 0);
  int sum = 0;
  if (v4) {
    q = in4(tid);
    sum = q.x + q.y + q.z + q.w;
  } else {
    for (int i = s0; i < s1; ++i) sum += in(i);
  }
  int x = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wtot[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int t = lane < LIST_WARPS ? wtot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < LIST_WARPS) wtot[lane] = t;
  }
  __syncthreads();
  int base = (warp ? wtot[warp - 1] : 0) + x - sum;
  if (v4) {
    reinterpret_cast<int4*>(out)[tid] = make_int4(base, base + q.x, base + q.x + q.y, base + q.x + q.y + q.z);
  } else {
    for (int i = s0; i < s1; ++i) {
      out[i] = base;
      base += in(i);
    }
  }
  const int total = wtot[LIST_WARPS - 1];
  __syncthreads();
  return total;
}

// The chunk's write ids and weights in shared memory with k = 16: (token t, write index i) is held at word
// t * 16 + (i ^ ((t >> 1) & 15)), a permutation within each token's row, so the 32 tokens of one write index (read
// together when the slot masks are built) fall in 32 distinct banks instead of two.  The map is its own inverse.
template <int K>
__device__ __forceinline__ int wslot(int e) {
  if constexpr (K == 16) return (e & ~15) | ((e & 15) ^ ((e >> 5) & 15));
  else return e;
}
// four consecutive elements u = 0..3 moved to positions u ^ m
template <typename V4>
__device__ __forceinline__ V4 perm4(V4 v, int m) {
  if (m & 1) v = V4{v.y, v.x, v.w, v.z};
  if (m & 2) v = V4{v.z, v.w, v.x, v.y};
  return v;
}

// ------------------------------------------------------------------------------------------------- list kernel
struct ListSmem {
  size_t siw, ww, sir, wr, V, run, pfx, tmask, ent, rst, wsl, lampow, prev_si, prev_w, prev_v, rec, misc, total;
};
__host__ __device__ inline ListSmem list_layout(int M, int k, int dh) {
  const int L = chunk_len(k), E = L * k;
  ListSmem s;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t r = o;
    o += align16(bytes);
    return r;
  };
  s.siw = take((size_t)E * 4);
  s.ww = take((size_t)E * 4);
  s.sir = take((size_t)E * 4);
  s.wr = take((size_t)E * 4);
  s.V = take((size_t)L * dh * 4);
  s.run = take((size_t)M * 4);
  s.tmask = take((size_t)M * 8);
  s.ent = take((size_t)E * 8);
  s.rst = take((size_t)L * 4);
  s.wsl = take((size_t)L * 4);
  s.lampow = take((size_t)(L + 1) * 4);
  s.prev_si = take((size_t)SCAN_MAX_K * 4);
  s.prev_w = take((size_t)SCAN_MAX_K * 4);
  s.prev_v = take((size_t)dh * 4);
  s.misc = take(64);
  // the record phase runs after the intra reads: its prefix sums reuse the write ids (dead once the entries are
  // built) and its staging reuses the values when they are large enough
  s.pfx = (size_t)E * 4 >= (size_t)M * 4 ? s.siw : take((size_t)M * 4);
  s.rec = (size_t)L * dh * 4 >= rec_layout(k).bytes ? s.V : take(rec_layout(k).bytes);
  s.total = o;
  return s;
}

// K: compile-time k (0: runtime).  DH: compile-time head width, a multiple of 32 (0: runtime, any width).
template <int K, int DH>
__global__ void __launch_bounds__(LIST_THREADS) rt_lists_kernel(ScanArgs a, int nch) {
  pdl_enter();
  extern __shared__ __align__(16) unsigned char smem[];
  const int k = K > 0 ? K : a.k;
  const int dh = DH > 0 ? DH : a.dh;
  const int M = a.M, h = a.h, T = a.T;
  const int L = chunk_len(k);
  const ListSmem lay = list_layout(M, k, dh);
  const RecLayout rl = rec_layout(k);
  int* siw_s = reinterpret_cast<int*>(smem + lay.siw);
  float* ww_s = reinterpret_cast<float*>(smem + lay.ww);
  int* sir_s = reinterpret_cast<int*>(smem + lay.sir);
  float* wr_s = reinterpret_cast<float*>(smem + lay.wr);
  float* V_s = reinterpret_cast<float*>(smem + lay.V);
  int* run = reinterpret_cast<int*>(smem + lay.run);  // slot r's entries: ent[run & 0xFFFF], run >> 16 of them
  int* pfx = reinterpret_cast<int*>(smem + lay.pfx);
  unsigned long long* tmask = reinterpret_cast<unsigned long long*>(smem + lay.tmask);  // tokens writing a slot
  int* cntt = reinterpret_cast<int*>(smem + lay.tmask);  // per-slot counts where tmask is not in use
  int2* ent = reinterpret_cast<int2*>(smem + lay.ent);  // entries by slot, then token: {slot << 16 | token, ww bits}
  int* rst_s = reinterpret_cast<int*>(smem + lay.rst);
  int* wsl = reinterpret_cast<int*>(smem + lay.wsl);
  float* lampow = reinterpret_cast<float*>(smem + lay.lampow);
  int* prev_si = reinterpret_cast<int*>(smem + lay.prev_si);
  float* prev_w = reinterpret_cast<float*>(smem + lay.prev_w);
  float* prev_v = reinterpret_cast<float*>(smem + lay.prev_v);
  unsigned char* rec_s = smem + lay.rec;
  int* misc = reinterpret_cast<int*>(smem + lay.misc);  // [0..8) scan totals, [8..11) chunk flags, [11] repeat

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned FULL = 0xffffffffu;
  const int c = blockIdx.x % nch;
  const int bh = blockIdx.x / nch;  // b * h + hh
  const int hh = bh % h, b = bh / h;
  const int c0 = c * L, Lc = min(L, T - c0), E = Lc * k;
  const float lam = a.decay[hh];
  const int mode = fade_mode(lam);
  const bool last_chunk = c == nch - 1;
  const int64_t sel0 = ((int64_t)bh * T + c0) * k;
  const int64_t tok0 = (int64_t)b * T + c0;
  const float* Vh = a.V + (int64_t)hh * dh;

  // ids outside [0, M) never come from the address kernel; they are clamped so no access leaves the state
  if ((E & 3) == 0 && ((reinterpret_cast<uintptr_t>(a.siw + sel0) | reinterpret_cast<uintptr_t>(a.ww + sel0) |
                        reinterpret_cast<uintptr_t>(a.sir + sel0) | reinterpret_cast<uintptr_t>(a.wr + sel0)) & 15) == 0) {
    for (int e4 = tid; e4 < E / 4; e4 += LIST_THREADS) {
      const int4 sw = reinterpret_cast<const int4*>(a.siw + sel0)[e4];
      const int4 sr = reinterpret_cast<const int4*>(a.sir + sel0)[e4];
      // k = 16: the four ids land permuted in one aligned group of the token's row (wslot)
      const int sq = K == 16 ? (e4 >> 3) & 15 : 0, d4 = (e4 & ~3) | ((e4 & 3) ^ (sq >> 2));
      reinterpret_cast<int4*>(siw_s)[d4] = perm4(make_int4(min(max(sw.x, 0), M - 1), min(max(sw.y, 0), M - 1),
                                                           min(max(sw.z, 0), M - 1), min(max(sw.w, 0), M - 1)),
                                                 sq & 3);
      reinterpret_cast<int4*>(sir_s)[e4] = make_int4(min(max(sr.x, 0), M - 1), min(max(sr.y, 0), M - 1),
                                                     min(max(sr.z, 0), M - 1), min(max(sr.w, 0), M - 1));
      reinterpret_cast<float4*>(ww_s)[d4] = perm4(reinterpret_cast<const float4*>(a.ww + sel0)[e4], sq & 3);
      reinterpret_cast<float4*>(wr_s)[e4] = reinterpret_cast<const float4*>(a.wr + sel0)[e4];
    }
  } else {
    for (int e = tid; e < E; e += LIST_THREADS) {
      siw_s[wslot<K>(e)] = min(max(a.siw[sel0 + e], 0), M - 1);
      ww_s[wslot<K>(e)] = a.ww[sel0 + e];
      sir_s[e] = min(max(a.sir[sel0 + e], 0), M - 1);
      wr_s[e] = a.wr[sel0 + e];
    }
  }
  if (DH > 0 && (a.ldv & 3) == 0 && (reinterpret_cast<uintptr_t>(Vh) & 15) == 0) {
    float4* V4 = reinterpret_cast<float4*>(V_s);
    for (int i = tid; i < Lc * (dh / 4); i += LIST_THREADS) {
      const int t = i / (dh / 4), q = i - t * (dh / 4);
      V4[i] = *reinterpret_cast<const float4*>(Vh + (tok0 + t) * a.ldv + 4 * q);
    }
  } else {
    for (int i = tid; i < Lc * dh; i += LIST_THREADS) {
      const int t = i / dh, col = i - t * dh;
      V_s[i] = Vh[(tok0 + t) * a.ldv + col];
    }
  }
  if (tid < L) rst_s[tid] = (a.reset && tid < Lc) ? (int)a.reset[tok0 + tid] : 0;
  if (tid <= L) lampow[tid] = mode == 0 ? (tid == 0 ? 1.f : 0.f) : powf(lam, (float)tid);
  if (mode == 0 && c0 > 0) {
    if (tid < k) {
      prev_si[tid] = min(max(a.siw[sel0 - k + tid], 0), M - 1);
      prev_w[tid] = a.ww[sel0 - k + tid];
    }
    for (int col = tid; col < dh; col += LIST_THREADS) prev_v[col] = Vh[(tok0 - 1) * a.ldv + col];
  }
  __syncthreads();
  // resets of the chunk (32 <= L <= 64): wsl[t] = last reset position <= t (-1: none), rd_end = first reset
  if (warp == 0) {
    const unsigned lo = __ballot_sync(FULL, rst_s[lane] != 0);
    const unsigned hi = __ballot_sync(FULL, 32 + lane < L && rst_s[min(32 + lane, L - 1)] != 0);
    const unsigned long long m = ((unsigned long long)hi << 32) | lo;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int t = lane + 32 * q;
      if (t < L) {
        const unsigned long long below = m & ((2ull << t) - 1ull);  // t = 63: 2ull << 63 wraps to 0, -1 = all ones
        wsl[t] = below ? 63 - __clzll((long long)below) : -1;
      }
    }
    if (lane == 0) {
      misc[8] = m ? __ffsll((long long)m) - 1 : Lc;    // rd_end
      misc[9] = m ? 1 : 0;                              // clear
      misc[10] = m ? 63 - __clzll((long long)m) : 0;   // first entry token of the state update
    }
  }
  __syncthreads();

  const bool need_sort = mode != 0 || last_chunk;
  if (need_sort) {
    // Group the entries by slot, in token order within a slot.  A token writes distinct slots, so the rank of an
    // entry in its slot's run is the number of earlier tokens of the chunk that wrote the slot: one bit per token.
    for (int r = tid; r < M; r += LIST_THREADS) tmask[r] = 0ull;
    if (tid == 0) misc[11] = 0;
    __syncthreads();
    // a warp takes one write index i of 32 consecutive tokens, so a slot that several of them write (repeated
    // tokens) is set by one atomic per warp: the lanes writing the same slot are matched and their token bits are
    // the matched lane mask shifted to the warp's first token
    for (int p = warp; p < k * 2; p += LIST_WARPS) {
      const int i = p % k, t = (p / k) * 32 + lane;
      const bool ok = t < Lc;
      const unsigned act = __ballot_sync(FULL, ok);
      if (ok) {
        const int r = siw_s[wslot<K>(t * k + i)];
        const unsigned peers = __match_any_sync(act, r);
        if (lane == __ffs(peers) - 1) {
          const unsigned long long bits = (unsigned long long)peers << ((p / k) * 32);
          const unsigned long long old = atomicOr(&tmask[r], bits);
          if (old & bits) misc[11] = 1;
        }
      }
    }
    __syncthreads();
    if (misc[11] == 0) {
      block_exclusive_scan([=](int r) { return __popcll(tmask[r]); },
                           [=](int g) {
                             const ulonglong2 m0 = reinterpret_cast<const ulonglong2*>(tmask)[2 * g];
                             const ulonglong2 m1 = reinterpret_cast<const ulonglong2*>(tmask)[2 * g + 1];
                             return make_int4(__popcll(m0.x), __popcll(m0.y), __popcll(m1.x), __popcll(m1.y));
                           },
                           run, M, misc);
#pragma unroll
      for (int q = 0; q < CH_MAX_E / LIST_THREADS; ++q) {
        const int e = tid + q * LIST_THREADS;
        if (e < E) {
          const int r = siw_s[e], t = e / k;
          ent[run[r] + __popcll(tmask[r] & ((1ull << t) - 1ull))] = make_int2((r << 16) | t, __float_as_int(ww_s[e]));
        }
      }
      __syncthreads();
      for (int r = tid; r < M; r += LIST_THREADS) run[r] |= __popcll(tmask[r]) << 16;
      __syncthreads();
    } else {
      // a token wrote one slot twice (ids from outside the address kernel): counting sort, then each run by entry
      for (int r = tid; r < M; r += LIST_THREADS) cntt[r] = 0;
      __syncthreads();
      int pos[CH_MAX_E / LIST_THREADS];
#pragma unroll
      for (int q = 0; q < CH_MAX_E / LIST_THREADS; ++q) {
        const int e = tid + q * LIST_THREADS;
        if (e < E) pos[q] = atomicAdd(&cntt[siw_s[e]], 1);
      }
      __syncthreads();
      block_exclusive_scan([=](int r) { return cntt[r]; },
                           [=](int g) { return reinterpret_cast<const int4*>(cntt)[g]; }, run, M, misc);
#pragma unroll
      for (int q = 0; q < CH_MAX_E / LIST_THREADS; ++q) {
        const int e = tid + q * LIST_THREADS;
        if (e < E) ent[run[siw_s[e]] + pos[q]] = make_int2(wslot<K>(e), __float_as_int(ww_s[e]));  // (t, i) order
      }
      __syncthreads();
      for (int r = tid; r < M; r += LIST_THREADS) {
        const int n = cntt[r], s0 = run[r];
        run[r] = s0 | (n << 16);
        for (int i = 1; i < n; ++i) {
          const int2 x = ent[s0 + i];
          int j = i - 1;
          while (j >= 0 && ent[s0 + j].x > x.x) {
            ent[s0 + j + 1] = ent[s0 + j];
            --j;
          }
          ent[s0 + j + 1] = x;
        }
      }
      __syncthreads();
      for (int x = tid; x < E; x += LIST_THREADS) ent[x].x = (siw_s[wslot<K>(ent[x].x)] << 16) | (ent[x].x / k);
      __syncthreads();
    }
  }

  // ---- intra-chunk reads
  if (mode == 0) {
    // only token t-1's writes are visible (none after a reset at t, none before the first token): warp per token
    for (int t = warp; t < Lc; t += LIST_WARPS) {
      const int ri = lane < k ? sir_s[t * k + lane] : -1;
      const float wi = lane < k ? wr_s[t * k + lane] : 0.f;
      if (t == 0 && c0 == 0 && a.mem_in) {
        // the window's first token reads the carried state unfaded (lam^0); nothing of it reaches later tokens
        const bool live = !rst_s[0];
        const float* mi = a.mem_in + (int64_t)bh * M * dh;
        const float dsum = live ? warp_sum(lane < k ? wi * a.cnt_in[(int64_t)bh * M + ri] : 0.f) : 0.f;
        float* dst = a.num + (tok0 * h + hh) * dh;
        for (int col = lane; col < dh; col += 32) {
          float acc = 0.f;
          for (int j = 0; j < k; ++j) acc = fmaf(wr_s[j], mi[(int64_t)sir_s[j] * dh + col], acc);
          dst[col] = live ? acc : 0.f;
        }
        if (lane == 0) a.den[tok0 * h + hh] = dsum;
        continue;
      }
      const bool has_src = !rst_s[t] && (t > 0 || c0 > 0);
      const float* sv = t > 0 ? V_s + (t - 1) * dh : prev_v;
      float dsum = 0.f;
      if (has_src) {
        const int* ssi = t > 0 ? siw_s + (t - 1) * k : prev_si;
        const float* sw = t > 0 ? ww_s + (t - 1) * k : prev_w;
        float m = 0.f;
        for (int j = 0; j < k; ++j) {
          const int jj = t > 0 ? wslot<K>((t - 1) * k + j) - (t - 1) * k : j;  // write index order
          if (ri == ssi[jj]) m += sw[jj];
        }
        dsum = warp_sum(wi * m);
      }
      const int64_t tok = tok0 + t;
      float* dst = a.num + (tok * h + hh) * dh;
      for (int col = lane; col < dh; col += 32) dst[col] = has_src ? dsum * sv[col] : 0.f;
      if (lane == 0) a.den[tok * h + hh] = dsum;
    }
  } else if constexpr (DH > 0) {
    // eight lanes per token: lane gl owns the float4 columns gl, gl + 8, ... of the head
    constexpr int NQ = DH / 32;
    const bool masks = misc[11] == 0;  // the per-slot token masks hold every entry (no token repeated a slot)
    const int grp = lane >> 3, gl = lane & 7;
    const float4* V4 = reinterpret_cast<const float4*>(V_s);
    const bool vst = (reinterpret_cast<uintptr_t>(a.num) & 15) == 0;
    for (int tb = warp * 4; tb < Lc; tb += LIST_WARPS * 4) {  // uniform per warp: every lane takes the shuffles
      const int t = tb + grp;
      const bool tv = t < Lc;  // a group past the chunk's end walks empty runs and stores nothing
      float4 acc[NQ];
#pragma unroll
      for (int q = 0; q < NQ; ++q) acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
      float dsum = 0.f;
      const int lo = tv ? max(wsl[t], 0) : 0;
      // lane gl of the token's group holds reads gl, gl + 8, ...: slot run (start | count << 16), the slot's
      // token mask and the read weight
      constexpr int NR = (K > 0 ? K : SCAN_MAX_K) / 8 > 0 ? (K > 0 ? K : SCAN_MAX_K) / 8 : 1;
      int rr[NR];
      unsigned long long rm[NR];
      float rw[NR];
#pragma unroll
      for (int m = 0; m < NR; ++m) {
        const int i = gl + 8 * m;
        const int r = (tv && i < k) ? sir_s[t * k + i] : -1;
        rr[m] = r >= 0 ? run[r] : 0;
        rm[m] = (r >= 0 && masks) ? tmask[r] : 0ull;
        rw[m] = r >= 0 ? wr_s[t * k + i] : 0.f;
      }
      // sources of token t: tokens lo .. t-1 of the chunk
      const unsigned long long win = tv ? (((1ull << t) - 1ull) & ~((1ull << lo) - 1ull)) : 0ull;
      for (int i = 0; i < k; ++i) {
        int ri = rr[0];
        unsigned long long mi = rm[0];
        float wi = rw[0];
#pragma unroll
        for (int m = 1; m < NR; ++m)
          if ((i >> 3) == m) {
            ri = rr[m];
            mi = rm[m];
            wi = rw[m];
          }
        const int src = (lane & 24) | (i & 7);
        const int rs = __shfl_sync(FULL, ri, src);
        const float w = __shfl_sync(FULL, wi, src);
        const int st = rs & 0xFFFF, en = st + (rs >> 16);
        if (masks) {
          // the slot's entries are in token order, so token s's entry sits at st + (earlier tokens in the mask)
          const unsigned long long tm = ((unsigned long long)__shfl_sync(FULL, (unsigned)(mi >> 32), src) << 32) |
                                        __shfl_sync(FULL, (unsigned)mi, src);
          unsigned long long mm = tm & win;
          while (mm) {
            const int s = __ffsll((long long)mm) - 1;
            mm &= mm - 1ull;
            const int2 q2 = ent[st + __popcll(tm & ((1ull << s) - 1ull))];
            const float cf = w * __int_as_float(q2.y) * lampow[t - 1 - s];
            dsum += cf;
#pragma unroll
            for (int q = 0; q < NQ; ++q) fma4(acc[q], cf, V4[s * (DH / 4) + gl + 8 * q]);
          }
        } else {
          // a token wrote one slot twice: walk the run (entries in token, then write order)
          for (int x = st; x < en; ++x) {
            const int2 q2 = ent[x];
            const int s = q2.x & 0xFFFF;
            if (s >= t) break;
            if (s < lo) continue;
            const float cf = w * __int_as_float(q2.y) * lampow[t - 1 - s];
            dsum += cf;
#pragma unroll
            for (int q = 0; q < NQ; ++q) fma4(acc[q], cf, V4[s * (DH / 4) + gl + 8 * q]);
          }
        }
      }
      if (!tv) continue;
      const int64_t tok = tok0 + t;
      float* dst = a.num + (tok * h + hh) * DH;
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        if (vst) {
          reinterpret_cast<float4*>(dst)[gl + 8 * q] = acc[q];
        } else {
          float* d1 = dst + 4 * (gl + 8 * q);
          d1[0] = acc[q].x;
          d1[1] = acc[q].y;
          d1[2] = acc[q].z;
          d1[3] = acc[q].w;
        }
      }
      if (gl == 0) a.den[tok * h + hh] = dsum;
    }
  } else {
    // any head width: warp per token, lanes over columns
    for (int t = warp; t < Lc; t += LIST_WARPS) {
      float acc[LIST_MAX_DH / 32];
#pragma unroll
      for (int q = 0; q < LIST_MAX_DH / 32; ++q) acc[q] = 0.f;
      float dsum = 0.f;
      const int ri = lane < k ? sir_s[t * k + lane] : -1;
      const float wi = lane < k ? wr_s[t * k + lane] : 0.f;
      const int lo = max(wsl[t], 0);
      const int st = ri >= 0 ? run[ri] & 0xFFFF : 0, n = ri >= 0 ? run[ri] >> 16 : 0;
      unsigned act = __ballot_sync(FULL, n > 0);
      while (act) {
        const int i = __ffs(act) - 1;
        act &= act - 1u;
        const int sti = __shfl_sync(FULL, st, i), ni = __shfl_sync(FULL, n, i);
        const float wii = __shfl_sync(FULL, wi, i);
        for (int x = sti; x < sti + ni; ++x) {
          const int2 q2 = ent[x];
          const int s = q2.x & 0xFFFF;
          if (s >= t) break;
          if (s < lo) continue;
          const float cf = wii * __int_as_float(q2.y) * lampow[t - 1 - s];
          dsum += cf;
#pragma unroll
          for (int q = 0; q < LIST_MAX_DH / 32; ++q) {
            const int col = lane + 32 * q;
            if (col < dh) acc[q] = fmaf(cf, V_s[s * dh + col], acc[q]);
          }
        }
      }
      const int64_t tok = tok0 + t;
      float* dst = a.num + (tok * h + hh) * dh;
#pragma unroll
      for (int q = 0; q < LIST_MAX_DH / 32; ++q) {
        const int col = lane + 32 * q;
        if (col < dh) dst[col] = acc[q];
      }
      if (lane == 0) a.den[tok * h + hh] = dsum;
    }
  }
  if (!need_sort) return;
  __syncthreads();

  // ---- the chunk record: entries from token p_first on, grouped by slot
  const int p_first = mode == 0 ? Lc - 1 : misc[10];
  for (int r = tid; r < M; r += LIST_THREADS) {
    const int n = run[r] >> 16, s0 = run[r] & 0xFFFF;
    int skip = 0;
    while (skip < n && (ent[s0 + skip].x & 0xFFFF) < p_first) ++skip;
    const int vc = n - skip;
    run[r] = s0 + skip;
    // packed counts for one prefix sum: entries (bits 0-10), jobs (11-21), long jobs (22-)
    cntt[r] = vc | (vc > 0 ? 1 << 11 : 0) | (vc >= kLongRun ? 1 << 22 : 0);
  }
  __syncthreads();
  const int tot = block_exclusive_scan([=](int r) { return cntt[r]; },
                                       [=](int g) { return reinterpret_cast<const int4*>(cntt)[g]; }, pfx, M, misc);
  const int nent = tot & 0x7FF, njobs = (tot >> 11) & 0x7FF, nlong = tot >> 22;
  int2* jobs_s = reinterpret_cast<int2*>(rec_s);
  int2* ents_s = reinterpret_cast<int2*>(rec_s + rl.ents);
  for (int r = tid; r < M; r += LIST_THREADS) {
    const int vc = cntt[r] & 0x7FF;
    if (vc) {
      const int p = pfx[r], eo = p & 0x7FF, pj = (p >> 11) & 0x7FF, pl = p >> 22;
      jobs_s[vc >= kLongRun ? pl : nlong + pj - pl] = make_int2(r, eo | (vc << 16));
    }
  }
  for (int x = tid; x < E; x += LIST_THREADS) {  // entry x of slot r's run goes to r's output block
    const int2 q2 = ent[x];
    const int r = (int)((unsigned)q2.x >> 16), t = q2.x & 0xFFFF, first = run[r];
    if (x >= first)
      ents_s[(pfx[r] & 0x7FF) + (x - first)] = make_int2(t, __float_as_int(__int_as_float(q2.y) * lampow[Lc - 1 - t]));
  }
  if (tid == 0) {
    reinterpret_cast<int4*>(a.rec + rec_region_bytes(a.B, T, h, k))[(int64_t)bh * nch + c] =
        make_int4(njobs, nent, misc[8], misc[9]);
  }
  __syncthreads();
  // copy out the used parts (16-byte stores)
  unsigned char* rec = a.rec + ((int64_t)bh * nch + c) * rl.bytes;
  const int n_jobs16 = (int)(align16((size_t)njobs * 8) / 16);
  const int n_ent16 = (int)(align16((size_t)nent * 8) / 16);
  for (int i = tid; i < n_jobs16 + n_ent16; i += LIST_THREADS) {
    const size_t o = i < n_jobs16 ? (size_t)i * 16 : rl.ents + (size_t)(i - n_jobs16) * 16;
    *reinterpret_cast<uint4*>(rec + o) = *reinterpret_cast<const uint4*>(rec_s + o);
  }
}

// ------------------------------------------------------------------------------------------------- state scan
struct ScanBuf {
  size_t hdr, rec, sir, wr, V, numi, deni, bytes;
};
__host__ __device__ inline ScanBuf scan_buf_layout(int k, int cw) {
  const int L = chunk_len(k), E = L * k;
  ScanBuf s;
  size_t o = 0;
  auto take = [&](size_t bytes) {  // 128-byte aligned: tensor-copy destinations
    const size_t r = o;
    o += (bytes + 127) & ~(size_t)127;
    return r;
  };
  s.hdr = take(16);
  s.rec = take(rec_layout(k).bytes);
  s.sir = take((size_t)E * 4);
  s.wr = take((size_t)E * 4);
  s.V = take((size_t)L * cw * 4);
  s.numi = take((size_t)L * cw * 4);
  s.deni = take((size_t)L * 4 * 4);  // TMA mode: a 4-head-wide box per token (the head's column at hh % 4)
  s.bytes = o;
  return s;
}
// P | Pc | two chunk buffers (128-byte aligned) | lampow, plus 128 bytes to align the dynamic region's base.
__host__ __device__ inline size_t scan_bufs_offset(int M, int cw) {
  return ((align16((size_t)M * cw * 4) + align16((size_t)M * 4)) + 127) & ~(size_t)127;
}
__host__ __device__ inline size_t scan_smem_bytes(int M, int k, int cw) {
  return 128 + scan_bufs_offset(M, cw) + 2 * scan_buf_layout(k, cw).bytes + align16((size_t)(CH_MAX_L + 1) * 4);
}

// Issue the cp.async copies of chunk c's inputs (header hd) into buffer `buf` (all threads).
__device__ __forceinline__ void scan_issue(const ScanArgs& a, unsigned char* buf, const ScanBuf& sb,
                                           const RecLayout& rl, int nch, int c, int4 hd, int b, int hh, int cs,
                                           int ncols, int cw, bool want_reads) {
  const int tid = threadIdx.x, k = a.k, h = a.h, dh = a.dh, T = a.T;
  const int L = chunk_len(k), c0 = c * L, Lc = min(L, T - c0), E = Lc * k;
  const int64_t bh = (int64_t)b * h + hh;
  const int64_t tok0 = (int64_t)b * T + c0;
  const unsigned char* rec = a.rec + (bh * nch + c) * rl.bytes;
  copy_words_async(buf + sb.rec, rec, 2 * hd.x, tid, SCAN_THREADS);
  copy_words_async(buf + sb.rec + rl.ents, rec + rl.ents, 2 * hd.y, tid, SCAN_THREADS);
  copy_rows32_async(buf + sb.V, a.V + tok0 * a.ldv + (int64_t)hh * dh + cs * cw, Lc, ncols, cw, a.ldv, tid,
                    SCAN_THREADS);
  if (want_reads && hd.z > 0) {
    const int64_t sel0 = (bh * T + c0) * k;
    const int nr = hd.z;  // tokens before the first reset read the state
    copy_words_async(buf + sb.sir, a.sir + sel0, nr * k, tid, SCAN_THREADS);
    copy_words_async(buf + sb.wr, a.wr + sel0, nr * k, tid, SCAN_THREADS);
    copy_rows32_async(buf + sb.numi, a.num + (tok0 * h + hh) * dh + cs * cw, nr, ncols, cw, (int64_t)h * dh, tid,
                      SCAN_THREADS);
    if (cs == 0) {
      float* dd = reinterpret_cast<float*>(buf + sb.deni);
      for (int i = tid; i < nr; i += SCAN_THREADS) cp_async4(dd + i, a.den + (tok0 + i) * h + hh);
    }
  }
  (void)E;
  cp_async_commit();
}

__device__ __forceinline__ void copy_rows32_async(void* dst, const void* src, int rows, int w, int cw, int64_t stride,
                                                  int tid, int nt) {
  const uint32_t* s = static_cast<const uint32_t*>(src);
  uint32_t* d = static_cast<uint32_t*>(dst);
  if (w == cw && (reinterpret_cast<uintptr_t>(s) & 15) == 0 && (stride & 3) == 0) {
    for (int i = tid; i < rows * (cw / 4); i += nt) {
      const int r = i / (cw / 4), q = i % (cw / 4);
      cp_async16(d + r * cw + 4 * q, s + r * stride + 4 * q);
    }
  } else {
    copy_rows_async(dst, src, rows, w, cw, stride, tid, nt);
  }
}

// Issue chunk c's inputs (header hd) into buffer `buf` with TMA, completing on `bar` (one thread).  Record parts and
// read selections are 1-D bulk copies of their exact (16-byte rounded) sizes; the value slice, intra num slice and
// the 4-head den box are 2-D tensor copies of L token rows.
__device__ __forceinline__ void scan_issue_tma(const ScanArgs& a, unsigned char* buf, uint64_t* bar,
                                               const ScanBuf& sb, const RecLayout& rl, int nch, int c, int4 hd,
                                               int b, int hh, int cs, int cw, bool want_reads, const CUtensorMap* mV,
                                               const CUtensorMap* mN, const CUtensorMap* mD) {
  const int k = a.k, h = a.h, dh = a.dh, T = a.T;
  const int L = chunk_len(k), c0 = c * L;
  const int64_t bh = (int64_t)b * h + hh;
  const unsigned char* rec = a.rec + (bh * nch + c) * rl.bytes;
  const uint32_t jb = (uint32_t)align16((size_t)hd.x * 8), eb = (uint32_t)align16((size_t)hd.y * 8);
  const int nr = want_reads ? hd.z : 0;
  const uint32_t selb = (uint32_t)nr * k * 4, slab = (uint32_t)L * cw * 4;
  uint32_t total = 16 + jb + eb + slab;
  if (nr > 0) total += 2 * selb + slab + (cs == 0 ? (uint32_t)L * 16 : 0u);
  tma::mbar_arrive_expect_tx(bar, total);
  tma::load_1d(buf + sb.hdr, reinterpret_cast<const int4*>(a.rec + rec_region_bytes(a.B, T, h, k)) + bh * nch + c,
               16, bar);
  if (jb) tma::load_1d(buf + sb.rec, rec, jb, bar);
  if (eb) tma::load_1d(buf + sb.rec + rl.ents, rec + rl.ents, eb, bar);
  const int x = hh * dh + cs * cw, y = b * T + c0;
  tma::load_2d(mV, bar, buf + sb.V, x, y);
  if (nr > 0) {
    const int64_t sel0 = (bh * T + c0) * k;
    tma::load_1d(buf + sb.sir, a.sir + sel0, selb, bar);
    tma::load_1d(buf + sb.wr, a.wr + sel0, selb, bar);
    tma::load_2d(mN, bar, buf + sb.numi, x, y);
    if (cs == 0) tma::load_2d(mD, bar, buf + sb.deni, hh & ~3, y);
  }
}

template <int K, int CW>
__global__ void __launch_bounds__(SCAN_THREADS, 1)
    rt_scan_kernel(ScanArgs a, int nch, int n_slices, const __grid_constant__ CUtensorMap mapV,
                   const __grid_constant__ CUtensorMap mapN, const __grid_constant__ CUtensorMap mapD, int use_tma) {
  pdl_enter();
  __shared__ __align__(8) uint64_t full_bar[2];
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~(uintptr_t)127);
  const int k = K > 0 ? K : a.k;
  constexpr int KR = K > 0 ? K : SCAN_MAX_K;
  constexpr int LPG = CW / 4, NG = 32 / LPG;  // lanes per group (one float4 each), groups per warp
  // vector reads: each token's reads in two halves, one lane group each (the same sums in the same order for
  // either slice width, so both give identical results), NG / 2 tokens per warp
  constexpr int NP = 2, TPW = NG / NP;
  constexpr bool kVecReads = K > 0 && K % (4 * NP) == 0;
  const int M = a.M, dh = a.dh, h = a.h, T = a.T;
  const int L = chunk_len(k);
  const RecLayout rl = rec_layout(k);
  const ScanBuf sb = scan_buf_layout(k, CW);
  float4* P4 = reinterpret_cast<float4*>(smem);
  float* P = reinterpret_cast<float*>(smem);
  float* Pc = reinterpret_cast<float*>(smem + align16((size_t)M * CW * 4));
  unsigned char* bufs = smem + scan_bufs_offset(M, CW);
  float* lampow = reinterpret_cast<float*>(bufs + 2 * sb.bytes);

  const int cs = blockIdx.x % n_slices;
  const int bh = blockIdx.x / n_slices;
  const int hh = bh % h, b = bh / h;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = lane / LPG, c4 = lane % LPG;
  const unsigned FULL = 0xffffffffu;
  const int ncols = min(CW, dh - cs * CW);
  const float lam = a.decay[hh];
  const int mode = fade_mode(lam);
  // fade 0: the intra pass already produced every read; only the final state (the last token's writes) is left
  if (mode == 0 && !a.mem_out && !a.cnt_out) return;
  const int c_begin = mode == 0 ? nch - 1 : 0;
  const bool reads = mode != 0;
  const int4* hdrs = reinterpret_cast<const int4*>(a.rec + rec_region_bytes(a.B, T, h, k)) + (int64_t)bh * nch;

  if (a.mem_in && mode != 0) {
    // the carried state (fade 0 keeps none of it past the first token, whose read the list kernel makes)
    const float* mi = a.mem_in + ((int64_t)b * h + hh) * (int64_t)M * dh + cs * CW;
    for (int i = tid; i < M * CW; i += SCAN_THREADS) {
      const int r = i / CW, cc = i % CW;
      P[i] = cc < ncols ? mi[(int64_t)r * dh + cc] : 0.f;
    }
    const float* ci = a.cnt_in + ((int64_t)b * h + hh) * (int64_t)M;
    for (int i = tid; i < M; i += SCAN_THREADS) Pc[i] = ci[i];
  } else {
    for (int i = tid; i < M * (CW / 4); i += SCAN_THREADS) P4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = tid; i < M; i += SCAN_THREADS) Pc[i] = 0.f;
  }
  if (ncols < CW) {  // columns past dh stay zero in both buffers (never copied, never stored)
    for (int i = tid; i < 2 * L * CW; i += SCAN_THREADS) {
      const int bb = i / (L * CW), j = i - bb * L * CW;
      reinterpret_cast<float*>(bufs + bb * sb.bytes + sb.V)[j] = 0.f;
      reinterpret_cast<float*>(bufs + bb * sb.bytes + sb.numi)[j] = 0.f;
    }
  }
  if (tid <= L) lampow[tid] = mode == 0 ? (tid == 0 ? 1.f : 0.f) : powf(lam, (float)tid);
  int4 hd = make_int4(0, 0, 0, 0), hd1 = hd;  // cp.async mode: this chunk's header and the next one's
  int4 hn = hd;                                // TMA mode (thread 0): the header of the next chunk to issue
  if (use_tma) {
    if (tid == 0) {
      tma::mbar_init(&full_bar[0], 1);
      tma::mbar_init(&full_bar[1], 1);
      tma::mbar_init_fence();
      tma::prefetch_map(&mapV);
      tma::prefetch_map(&mapN);
      tma::prefetch_map(&mapD);
    }
    __syncthreads();
    if (tid == 0) {
      scan_issue_tma(a, bufs, &full_bar[0], sb, rl, nch, c_begin, hdrs[c_begin], b, hh, cs, CW, reads, &mapV, &mapN,
                     &mapD);
      if (c_begin + 1 < nch) hn = hdrs[c_begin + 1];
    }
  } else {
    hd = hdrs[c_begin];
    hd1 = c_begin + 1 < nch ? hdrs[c_begin + 1] : make_int4(0, 0, 0, 0);
    __syncthreads();
    scan_issue(a, bufs, sb, rl, nch, c_begin, hd, b, hh, cs, ncols, CW, reads);
  }

  float sigma = 1.f;  // state = sigma * P
  int buf = 0;
  for (int c = c_begin; c < nch; ++c, buf ^= 1) {
    unsigned char* cur = bufs + buf * sb.bytes;
    int4 hd2 = make_int4(0, 0, 0, 0);
    if (use_tma) {
      // every thread waits for this chunk's copies (bounded); a wait that gave up ends the CTA on all threads
      const bool ok = tma::mbar_wait(&full_bar[buf], (uint32_t)((c - c_begin) >> 1) & 1u);
      if (__syncthreads_or(!ok)) {
        if (ok == false) tma::mbar_wait(&full_bar[buf], (uint32_t)((c - c_begin) >> 1) & 1u);  // drain, bounded
        return;
      }
      hd = *reinterpret_cast<const int4*>(cur + sb.hdr);
    } else {
      cp_async_wait_all();
      __syncthreads();
      if (c + 1 < nch) scan_issue(a, bufs + (buf ^ 1) * sb.bytes, sb, rl, nch, c + 1, hd1, b, hh, cs, ncols, CW, reads);
      hd2 = c + 2 < nch ? hdrs[c + 2] : make_int4(0, 0, 0, 0);  // used two iterations on
    }
    const int njobs = hd.x, rd_end = hd.z, clear = hd.w;
    const int c0 = c * L, Lc = min(L, T - c0);
    const float4* V4 = reinterpret_cast<const float4*>(cur + sb.V);

    if (reads) {
      const int* sir_b = reinterpret_cast<const int*>(cur + sb.sir);
      const float* wr_b = reinterpret_cast<const float*>(cur + sb.wr);
      const float4* numi4 = reinterpret_cast<const float4*>(cur + sb.numi);
      const float* deni = reinterpret_cast<const float*>(cur + sb.deni);
      const int dstr = use_tma ? 4 : 1, doff = use_tma ? (hh & 3) : 0;  // den of token t at deni[t * dstr + doff]
      const float sg = mode == 2 ? sigma : 1.f;
      if constexpr (kVecReads) {
        // two lane groups per token (reads [0, K/2) and [K/2, K)), TPW tokens per warp; read ids and weights four
        // at a time; the halves are combined with one shuffle (the loop is warp-uniform, so every lane takes it)
        const int half = grp % NP;
        for (int tb = TPW * warp; tb < rd_end; tb += TPW * SCAN_WARPS) {
          const int t = tb + grp / NP;
          const bool tv = t < rd_end;
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          float dc = 0.f;
          if (tv) {
            const int4* s4 = reinterpret_cast<const int4*>(sir_b + t * K + half * (K / NP));
            const float4* w4 = reinterpret_cast<const float4*>(wr_b + t * K + half * (K / NP));
#pragma unroll
            for (int q = 0; q < K / (4 * NP); ++q) {
              const int4 rr = s4[q];
              const float4 wv = w4[q];
              const int r0 = min(max(rr.x, 0), M - 1), r1 = min(max(rr.y, 0), M - 1);
              const int r2 = min(max(rr.z, 0), M - 1), r3 = min(max(rr.w, 0), M - 1);
              fma4(acc, wv.x, P4[r0 * (CW / 4) + c4]);
              fma4(acc, wv.y, P4[r1 * (CW / 4) + c4]);
              fma4(acc, wv.z, P4[r2 * (CW / 4) + c4]);
              fma4(acc, wv.w, P4[r3 * (CW / 4) + c4]);
              dc = fmaf(wv.x, Pc[r0], dc);
              dc = fmaf(wv.y, Pc[r1], dc);
              dc = fmaf(wv.z, Pc[r2], dc);
              dc = fmaf(wv.w, Pc[r3], dc);
            }
          }
          acc.x += __shfl_xor_sync(FULL, acc.x, LPG);
          acc.y += __shfl_xor_sync(FULL, acc.y, LPG);
          acc.z += __shfl_xor_sync(FULL, acc.z, LPG);
          acc.w += __shfl_xor_sync(FULL, acc.w, LPG);
          dc += __shfl_xor_sync(FULL, dc, LPG);
          if (!tv) continue;
          const float fade = sg * lampow[t];
          const int64_t tok = (int64_t)b * T + c0 + t;
          if (half == 0) {
            const float4 ni = numi4[t * (CW / 4) + c4];
            const float o0 = fmaf(fade, acc.x, ni.x), o1 = fmaf(fade, acc.y, ni.y);
            const float o2 = fmaf(fade, acc.z, ni.z), o3 = fmaf(fade, acc.w, ni.w);
            float* dst = a.num + (tok * h + hh) * dh + cs * CW + 4 * c4;
            if (4 * c4 + 3 < ncols && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
              *reinterpret_cast<float4*>(dst) = make_float4(o0, o1, o2, o3);
            } else {
              if (4 * c4 + 0 < ncols) dst[0] = o0;
              if (4 * c4 + 1 < ncols) dst[1] = o1;
              if (4 * c4 + 2 < ncols) dst[2] = o2;
              if (4 * c4 + 3 < ncols) dst[3] = o3;
            }
          } else if (cs == 0 && c4 == 0) {
            a.den[tok * h + hh] = fmaf(fade, dc, deni[t * dstr + doff]);
          }
        }
      } else {
        // any k: warp per token, the NG lane groups take reads g, g + NG, ...
        for (int t = warp; t < rd_end; t += SCAN_WARPS) {
          int ri = 0;
          float wi = 0.f, pdi = 0.f;
          if (lane < k) {
            ri = min(max(sir_b[t * k + lane], 0), M - 1);
            wi = wr_b[t * k + lane];
            pdi = Pc[ri];
          }
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int q = 0; q < (KR + NG - 1) / NG; ++q) {
            const int ii = NG * q + grp;
            const int r = __shfl_sync(FULL, ri, ii & 31);
            const float w = __shfl_sync(FULL, wi, ii & 31);
            if (ii < k) fma4(acc, w, P4[r * (CW / 4) + c4]);
          }
#pragma unroll
          for (int o = LPG; o < 32; o <<= 1) {
            acc.x += __shfl_xor_sync(FULL, acc.x, o);
            acc.y += __shfl_xor_sync(FULL, acc.y, o);
            acc.z += __shfl_xor_sync(FULL, acc.z, o);
            acc.w += __shfl_xor_sync(FULL, acc.w, o);
          }
          const float dcar = warp_sum(wi * pdi);
          const float fade = sg * lampow[t];
          const int64_t tok = (int64_t)b * T + c0 + t;
          if (grp == 0) {
            const float4 ni = numi4[t * (CW / 4) + c4];
            const float o0 = fmaf(fade, acc.x, ni.x), o1 = fmaf(fade, acc.y, ni.y);
            const float o2 = fmaf(fade, acc.z, ni.z), o3 = fmaf(fade, acc.w, ni.w);
            float* dst = a.num + (tok * h + hh) * dh + cs * CW + 4 * c4;
            if (4 * c4 + 0 < ncols) dst[0] = o0;
            if (4 * c4 + 1 < ncols) dst[1] = o1;
            if (4 * c4 + 2 < ncols) dst[2] = o2;
            if (4 * c4 + 3 < ncols) dst[3] = o3;
          }
          if (cs == 0 && lane == 0) a.den[tok * h + hh] = fmaf(fade, dcar, deni[t * dstr + doff]);
        }
      }
    }
    __syncthreads();

    // the state after the chunk: a reset (or fade 0) empties it first, a tiny scale is folded into it
    float inv = 1.f;
    bool pass = false;
    float f = 0.f;
    if (mode == 0) {
      sigma = 1.f;  // only the last chunk runs, on the zero state
    } else if (clear) {
      pass = true;
      sigma = 1.f;
    } else if (mode == 2) {
      const float s2 = sigma * lampow[Lc];
      if (s2 < kRenorm) {
        pass = true;
        f = s2;
        sigma = 1.f;
      } else {
        sigma = s2;
        inv = 1.f / s2;
      }
    }
    if (pass) {
      for (int i = tid; i < M * (CW / 4); i += SCAN_THREADS) {
        const float4 v = P4[i];
        P4[i] = make_float4(v.x * f, v.y * f, v.z * f, v.w * f);
      }
      for (int i = tid; i < M; i += SCAN_THREADS) Pc[i] *= f;
      __syncthreads();
    }
    // writes: one lane group per written slot, NG slots per warp.  In TMA mode warp 0 instead issues the next
    // chunk's copies (each TMA instruction holds its thread for hundreds of cycles); their buffer has been free
    // since this chunk's first barrier.
    const int2* jobs = reinterpret_cast<const int2*>(cur + sb.rec);
    const int2* ents = reinterpret_cast<const int2*>(cur + sb.rec + rl.ents);
    const int wwarp = use_tma ? warp - 1 : warp, nww = use_tma ? SCAN_WARPS - 1 : SCAN_WARPS;
    if (use_tma && warp == 0) {
      if (lane == 0 && c + 1 < nch) {
        tma::fence_proxy_async();
        scan_issue_tma(a, bufs + (buf ^ 1) * sb.bytes, &full_bar[buf ^ 1], sb, rl, nch, c + 1, hn, b, hh, cs, CW,
                       reads, &mapV, &mapN, &mapD);
        if (c + 2 < nch) hn = hdrs[c + 2];
      }
      __syncwarp();
    }
    for (int jb = NG * wwarp; wwarp >= 0 && jb < njobs; jb += NG * nww) {
      const int j = jb + grp;
      if (j >= njobs) continue;
      const int2 jj = jobs[j];
      const int r = jj.x, st = jj.y & 0xFFFF, en = st + (jj.y >> 16);
      float4 d = make_float4(0.f, 0.f, 0.f, 0.f);
      float dc = 0.f;
#pragma unroll 2
      for (int e = st; e < en; ++e) {
        const int2 q2 = ents[e];
        const float cf = __int_as_float(q2.y);
        fma4(d, cf, V4[q2.x * (CW / 4) + c4]);
        dc += cf;
      }
      float4 p = P4[r * (CW / 4) + c4];
      fma4(p, inv, d);
      P4[r * (CW / 4) + c4] = p;
      if (c4 == 0) Pc[r] = fmaf(inv, dc, Pc[r]);
    }
    hd = hd1;
    hd1 = hd2;
  }
  __syncthreads();
  // the final state, unscaled
  const float fs = sigma;
  if (a.mem_out) {
    float* mo = a.mem_out + ((int64_t)b * h + hh) * (int64_t)M * dh;
    for (int i = tid; i < M * CW; i += SCAN_THREADS) {
      const int r = i / CW, cc = i % CW, gc = cs * CW + cc;
      if (gc < dh) mo[(int64_t)r * dh + gc] = P[i] * fs;
    }
  }
  if (a.cnt_out && cs == 0) {
    float* co = a.cnt_out + ((int64_t)b * h + hh) * (int64_t)M;
    for (int r = tid; r < M; r += SCAN_THREADS) co[r] = Pc[r] * fs;
  }
}

bool rt_scan_supported(int M, int dh, int k) {
  if (M < 1 || M > 65535 || dh < 1 || dh > LIST_MAX_DH || k < 1 || k > SCAN_MAX_K) return false;
  return scan_smem_bytes(M, k, SCAN_CW) <= 227 * 1024 && list_layout(M, k, dh).total <= 227 * 1024;
}

size_t rt_scan_workspace_bytes(int B, int T, int h, int k) {
  if (B <= 0 || T <= 0 || h <= 0 || k <= 0) return 0;
  const int L = chunk_len(k);
  return rec_region_bytes(B, T, h, k) + (size_t)B * h * ((T + L - 1) / L) * 16;  // records + headers
}

struct ScanMaps {
  CUtensorMap v, num, den;
  int use_tma;
};

// TMA staging of the scan's chunk inputs: value and num slices of cw columns (dh a multiple of cw), 1-D selection
// copies (k a multiple of 4), the 4-head den box (h a multiple of 4); else cp.async.
static ScanMaps scan_maps(const ScanArgs& a, int cw) {
  ScanMaps m{};
  const int L = chunk_len(a.k);
  const uint64_t rows = (uint64_t)a.B * a.T;
  const bool shape_ok = a.dh % cw == 0 && a.k % 4 == 0 && a.h % 4 == 0 && (a.ldv % 4) == 0 &&
                        ((reinterpret_cast<uintptr_t>(a.sir) | reinterpret_cast<uintptr_t>(a.wr) |
                          reinterpret_cast<uintptr_t>(a.V) | reinterpret_cast<uintptr_t>(a.num) |
                          reinterpret_cast<uintptr_t>(a.den)) & 15) == 0;
  m.use_tma = shape_ok &&
              make_tensor_map_2d(&m.v, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.V, (uint64_t)a.h * a.dh, rows,
                                 (uint64_t)a.ldv * 4, (uint32_t)cw, L, CU_TENSOR_MAP_SWIZZLE_NONE) &&
              make_tensor_map_2d(&m.num, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.num, (uint64_t)a.h * a.dh, rows,
                                 (uint64_t)a.h * a.dh * 4, (uint32_t)cw, L, CU_TENSOR_MAP_SWIZZLE_NONE) &&
              make_tensor_map_2d(&m.den, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a.den, (uint64_t)a.h, rows,
                                 (uint64_t)a.h * 4, 4, L, CU_TENSOR_MAP_SWIZZLE_NONE);
  return m;
}

static int scan_num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    cached[dev] = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0 ? n : 148;
  }
  return cached[dev];
}

template <int K, int CW>
static cudaError_t launch_state_scan(const ScanArgs& a, int nch, cudaStream_t st) {
  const size_t ssm = scan_smem_bytes(a.M, a.k, CW);
  cudaError_t e = cudaFuncSetAttribute(rt_scan_kernel<K, CW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ssm);
  if (e != cudaSuccess) return e;
  const int n_slices = (a.dh + CW - 1) / CW;
  const ScanMaps m = scan_maps(a, CW);
  LaunchScope scope_("rt_scan", st);
  return launch_k(rt_scan_kernel<K, CW>, dim3((unsigned)((int64_t)a.B * a.h * n_slices)), dim3(SCAN_THREADS), ssm, st,
                  a, nch, n_slices, m.v, m.num, m.den, m.use_tma);
}

template <int K, int DH>
static cudaError_t launch_scan_k(const ScanArgs& a, int nch, cudaStream_t st) {
  const size_t lsm = list_layout(a.M, a.k, a.dh).total;
  cudaError_t e =
      cudaFuncSetAttribute(rt_lists_kernel<K, DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lsm);
  if (e != cudaSuccess) return e;
  {
    LaunchScope scope_("rt_lists", st);
    launch_k(rt_lists_kernel<K, DH>, dim3((unsigned)((int64_t)a.B * a.h * nch)), dim3(LIST_THREADS), lsm, st, a, nch);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  // Each state CTA holds an SM for the whole window: when the 32-column slices of this launch would occupy at most
  // half the SMs (a few rows per GPU), 16-column slices halve each CTA's shared-memory work and use twice the SMs.
  if constexpr (K == 16) {
    const int64_t ctas32 = (int64_t)a.B * a.h * ((a.dh + SCAN_CW - 1) / SCAN_CW);
    if (2 * ctas32 <= scan_num_sms() && scan_smem_bytes(a.M, a.k, SCAN_CW_SMALL) <= 227 * 1024)
      return launch_state_scan<K, SCAN_CW_SMALL>(a, nch, st);
  }
  return launch_state_scan<K, SCAN_CW>(a, nch, st);
}

cudaError_t launch_rt_scan(const ScanArgs& a, cudaStream_t st) {
  if (a.B == 0 || a.T == 0) return cudaSuccess;
  if (!a.rec || !rt_scan_supported(a.M, a.dh, a.k)) return cudaErrorInvalidValue;
  const int nch = (a.T + chunk_len(a.k) - 1) / chunk_len(a.k);
  if (a.k == 16 && a.dh == 64) return launch_scan_k<16, 64>(a, nch, st);
  switch (a.k) {
    case 16: return launch_scan_k<16, 0>(a, nch, st);
    case 4: return launch_scan_k<4, 0>(a, nch, st);
    default: return launch_scan_k<0, 0>(a, nch, st);
  }
}

// Read and clear the bounded-wait timeout flag of the scan module.
cudaError_t read_and_clear_scan_timeout(int* flag, cudaStream_t st) {
  return tma::read_and_clear_wait_timeout(flag, st);
}
cudaError_t set_scan_wait_limit(unsigned long long ns) { return tma::set_wait_limit(ns); }

}  // namespace sdm
