// Product-key addressing on CUDA cores, float32-exact (track4_onesdm_models.py:134-148, soft weights :203-206).
//
// One thread owns one (token, head) address.  The address halves are L2-normalised, scored against the head's
// normalised sub-keys (kept in shared memory), and each half's top-c1 is found with a register bitonic network
// over 64-bit keys that encode the total order (score descending, sub-key index ascending).  The c1 x c1 cartesian combine is never
// built: a frontier walk over the two sorted lists emits the top-kk combined scores in (score descending,
// flat index a*c1+b ascending) order, which is the order a stable top-k of the reference's flattened `comb`
// gives.  Only exactly equal scores can order differently from aten::topk, whose tie order is unspecified.
#include "pk_common.cuh"
#include "tma.cuh"

namespace sdm {

__device__ __forceinline__ bool better(float va, int ia, float vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

// Sort C (power of two) keys descending: a bitonic network of max/min pairs (directions fixed at compile time).
template <int C>
__device__ __forceinline__ void bitonic_sort_desc(KT (&k)[C]) {
#pragma unroll
  for (int size = 2; size <= C; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < C; ++i) {
        const int j = i ^ stride;
        if (j > i) {
          const KT hi = kmax(k[i], k[j]), lo = kmin(k[i], k[j]);
          const bool desc = (i & size) == 0;
          k[i] = desc ? hi : lo;
          k[j] = desc ? lo : hi;
        }
      }
    }
  }
}

// t <- top-C of (t U g), both sorted descending; result sorted descending.
template <int C>
__device__ __forceinline__ void merge_top(KT (&t)[C], const KT (&g)[C]) {
#pragma unroll
  for (int q = 0; q < C; ++q) t[q] = kmax(t[q], g[C - 1 - q]);
#pragma unroll
  for (int stride = C >> 1; stride > 0; stride >>= 1) {
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int j = i ^ stride;
      if (j > i) {
        const KT hi = kmax(t[i], t[j]), lo = kmin(t[i], t[j]);
        t[i] = hi;
        t[j] = lo;
      }
    }
  }
}

// Top-C keys of the n_sub cosine scores of one normalised half against the sub-keys kn (n_sub, HALF) in shared
// memory; a NaN score orders last and padding entries (j >= n_sub) after every real one.
template <int HALF, int C>
__device__ __forceinline__ void half_topc(const float (&zn)[HALF], const float* kn, int n_sub, KT (&tk)[C]) {
  for (int g0 = 0; g0 < n_sub; g0 += C) {
    KT gk[C];
#pragma unroll
    for (int q = 0; q < C; ++q) {
      const int j = g0 + q;
      float s = -INFINITY;
      if (j < n_sub) {
        s = half_dot<HALF>(zn, kn + j * HALF);
        if (s != s) s = -INFINITY;
      }
      gk[q] = pk_key(s, j < n_sub ? (uint32_t)j : 0xFFFFFFFFu);
    }
    bitonic_sort_desc<C>(gk);
    if (g0 == 0) {
#pragma unroll
      for (int q = 0; q < C; ++q) tk[q] = gk[q];
    } else {
      merge_top<C>(tk, gk);
    }
  }
}

// Fast path (n_sub <= 32): 32-bit keys = the score's order-preserving image with its low 5 bits replaced by
// 31 - index, so one unsigned min and one max make a compare-exchange.  Their order can differ from the exact one
// only between two keys with equal high 27 bits (scores within ~2^-18 relative, or exactly tied); such a pair
// among the top C, or at the boundary to the best key left out, is detected and the half is re-sorted exactly.
constexpr int FK_IB = 5;
constexpr uint32_t FK_MASK = (1u << FK_IB) - 1u;
__device__ __forceinline__ uint32_t fast_key(float s, uint32_t j) {
  const uint32_t b = __float_as_uint(s + 0.f);
  const uint32_t m = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (m & ~FK_MASK) | (FK_MASK - j);
}
// Batcher's odd-even merge sort network on C keys (C a power of two): comparator I as (a, b), a < b, the larger key
// to a.  63 comparators for 16 keys and 191 for 32, against 80 and 240 in a bitonic network; evaluated at compile
// time, so every comparator is a pair of fixed registers.
constexpr int oe_pair(int C, int idx) {  // comparator idx packed as a * 256 + b; -1 past the last; the count at -1
  int n = 0;
  for (int p = 1; p < C; p <<= 1)
    for (int kk = p; kk >= 1; kk >>= 1)
      for (int j = kk % p; j + kk < C; j += 2 * kk)
        for (int i = 0; i < kk; ++i) {
          const int a = i + j, b = i + j + kk;
          if (b < C && a / (2 * p) == b / (2 * p)) {
            if (n == idx) return a * 256 + b;
            ++n;
          }
        }
  return idx < 0 ? n : -1;
}
template <int C, int I>
__device__ __forceinline__ void oe_apply(uint32_t (&k)[C]) {
  if constexpr (I < oe_pair(C, -1)) {
    constexpr int pr = oe_pair(C, I), a = pr >> 8, b = pr & 255;
    const uint32_t hi = max(k[a], k[b]), lo = min(k[a], k[b]);
    k[a] = hi;
    k[b] = lo;
    oe_apply<C, I + 1>(k);
  }
}
// k[0..C) sorted descending; the keys are distinct, so any sorting network gives the same order.
template <int C>
__device__ __forceinline__ void bitonic_sort_desc32(uint32_t (&k)[C]) {
  oe_apply<C, 0>(k);
}
// Sort only k[0..NS) descending (NS a power of two dividing C); entries past NS are left as they are.
template <int C, int NS>
__device__ __forceinline__ void bitonic_sort_desc32_head(uint32_t (&k)[C]) {
#pragma unroll
  for (int size = 2; size <= NS; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < NS; ++i) {
        const int j = i ^ stride;
        if (j > i) {
          const uint32_t hi = max(k[i], k[j]), lo = min(k[i], k[j]);
          const bool desc = (i & size) == 0;
          k[i] = desc ? hi : lo;
          k[j] = desc ? lo : hi;
        }
      }
    }
  }
}
// t <- top-C of (t U g); disc <- max(disc, the best key left out).
template <int C>
__device__ __forceinline__ void merge_top32(uint32_t (&t)[C], const uint32_t (&g)[C], uint32_t& disc) {
#pragma unroll
  for (int q = 0; q < C; ++q) {
    const uint32_t a = t[q], b = g[C - 1 - q];
    t[q] = max(a, b);
    disc = max(disc, min(a, b));
  }
#pragma unroll
  for (int stride = C >> 1; stride > 0; stride >>= 1) {
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int j = i ^ stride;
      if (j > i) {
        const uint32_t hi = max(t[i], t[j]), lo = min(t[i], t[j]);
        t[i] = hi;
        t[j] = lo;
      }
    }
  }
}
// Top-C of one half with 32-bit keys; the exact scores go to sc[j * PK_STRIDE].  False when the result may
// differ from the exact order (the caller then sorts the stored scores with 64-bit keys).
template <int HALF, int C, int PK_STRIDE>
__device__ __forceinline__ bool half_topc_fast(const float (&zn)[HALF], const float* kn, int n_sub, float* sc,
                                               uint32_t (&tk)[C]) {
  uint32_t disc = 0u;
  for (int g0 = 0; g0 < n_sub; g0 += C) {
    uint32_t gk[C];
#pragma unroll
    for (int q = 0; q < C; ++q) {
      const int j = g0 + q;
      uint32_t key = 0u;  // padding: below every real key
      if (j < n_sub) {
        float s = half_dot<HALF>(zn, kn + j * HALF);
        if (s != s) s = -INFINITY;
        sc[j * PK_STRIDE] = s;
        key = fast_key(s, (uint32_t)j);
      }
      gk[q] = key;
    }
    bitonic_sort_desc32<C>(gk);
    if (g0 == 0) {
#pragma unroll
      for (int q = 0; q < C; ++q) tk[q] = gk[q];
    } else {
      merge_top32<C>(tk, gk, disc);
    }
  }
  bool amb = disc != 0u && tk[C - 1] != 0u && (disc >> FK_IB) == (tk[C - 1] >> FK_IB);
#pragma unroll
  for (int q = 0; q + 1 < C; ++q) amb |= tk[q + 1] != 0u && (tk[q] >> FK_IB) == (tk[q + 1] >> FK_IB);
  return !amb;
}
// The exact top-C (64-bit keys) of scores already stored at sc[j * PK_STRIDE].
template <int C, int PK_STRIDE>
__device__ __noinline__ void half_topc_stored(const float* sc, int n_sub, KT (&tk)[C]) {
  for (int g0 = 0; g0 < n_sub; g0 += C) {
    KT gk[C];
#pragma unroll
    for (int q = 0; q < C; ++q) {
      const int j = g0 + q;
      gk[q] = j < n_sub ? pk_key(sc[j * PK_STRIDE], (uint32_t)j) : pk_key(-INFINITY, 0xFFFFFFFFu);
    }
    bitonic_sort_desc<C>(gk);
    if (g0 == 0) {
#pragma unroll
      for (int q = 0; q < C; ++q) tk[q] = gk[q];
    } else {
      merge_top<C>(tk, gk);
    }
  }
}

constexpr int PK_THREADS = 128;

// The top-kk of the c1 x c1 grid of combined scores (v1[a] + v2[b]) / 2 over two lists sorted descending, in
// (score descending, flat index a * c1 + b ascending) order: a frontier walk, row a's next candidate being
// (a, b_a).  The lists (value, sub-key id) live at v1s/i1s, v2s/i2s with stride PK_THREADS; the picks go to
// ov (combined score) and oi (slot id a' * n_sub + b') rows.
//
// walk_rows, for kk <= c1 (no row runs out of candidates before the walk ends): row q's first candidate ranks
// after row q-1's (the lists are sorted and rounding is monotone; equal scores go to the lower flat index), so at
// step s the largest candidate is in rows 0..s and the step's max tree spans s + 1 rows.  Between rows, flat
// index order is row order, so float compares with ties kept by the lower row give the exact order.
// One step (S, a compile-time constant, so every register index below is one too).
template <int C, int S>
__device__ __forceinline__ void walk_rows_step(float (&kv)[C], int (&kp)[C], const float* v1s, const int* i1s,
                                               const float* v2s, const int* i2s, float* ov, int* oi, int kk,
                                               int n_sub, int tid) {
  if constexpr (S < C) {
    if (S >= kk) return;
    float tv[S + 1];
    int tp[S + 1];
#pragma unroll
    for (int q = 0; q <= S; ++q) {
      tv[q] = kv[q];
      tp[q] = kp[q];
    }
#pragma unroll
    for (int w = 1; w <= S; w <<= 1) {
#pragma unroll
      for (int q = 0; q + w <= S; q += 2 * w) {
        const bool hi = tv[q + w] > tv[q];  // the higher rows' candidate only when strictly larger
        tv[q] = hi ? tv[q + w] : tv[q];
        tp[q] = hi ? tp[q + w] : tp[q];
      }
    }
    const int r = tp[0] >> 8, b = tp[0] & 255;
    ov[S * PK_THREADS + tid] = tv[0] + 0.f;  // -0 -> +0
    oi[S * PK_THREADS + tid] = i1s[r * PK_THREADS + tid] * n_sub + i2s[b * PK_THREADS + tid];
    const int nb = min(b + 1, C - 1);  // b + 1 = c1 only after the last pick
    const float nk = (v1s[r * PK_THREADS + tid] + v2s[nb * PK_THREADS + tid]) * 0.5f;
#pragma unroll
    for (int q = 0; q <= S; ++q) {
      const bool mine = q == r;
      kv[q] = mine ? nk : kv[q];
      kp[q] = mine ? kp[q] + 1 : kp[q];
    }
    walk_rows_step<C, S + 1>(kv, kp, v1s, i1s, v2s, i2s, ov, oi, kk, n_sub, tid);
  }
}
template <int C>
__device__ __forceinline__ void walk_rows(const float* v1s, const int* i1s, const float* v2s, const int* i2s,
                                          float* ov, int* oi, int kk, int n_sub, int tid) {
  float kv[C];
  int kp[C];  // row q's current candidate: q << 8 | b
  const float v2_0 = v2s[tid];
#pragma unroll
  for (int q = 0; q < C; ++q) {
    kv[q] = (v1s[q * PK_THREADS + tid] + v2_0) * 0.5f;
    kp[q] = q << 8;
  }
  walk_rows_step<C, 0>(kv, kp, v1s, i1s, v2s, i2s, ov, oi, kk, n_sub, tid);
}

// walk_keys, any kk <= c1 * c1: the candidates as 64-bit keys (tie r << 6 | b_r, which orders like the flat
// index); a row that runs out holds the key below every real one; each step takes the largest key of all C rows.
template <int C>
__device__ __forceinline__ void walk_keys(const float* v1s, const int* i1s, const float* v2s, const int* i2s,
                                          float* ov, int* oi, int c1, int kk, int n_sub, int tid) {
  KT kq[C];
  const float v2_0 = v2s[tid];
  const KT kminv = pk_key(-INFINITY, 0xFFFFFFFFu);
#pragma unroll
  for (int q = 0; q < C; ++q)
    kq[q] = q < c1 ? pk_key((v1s[q * PK_THREADS + tid] + v2_0) * 0.5f, (uint32_t)(q << 6)) : kminv;
  for (int step = 0; step < kk; ++step) {
    KT t[C];
#pragma unroll
    for (int q = 0; q < C; ++q) t[q] = kq[q];
#pragma unroll
    for (int w = C / 2; w >= 1; w >>= 1) {
#pragma unroll
      for (int q = 0; q < w; ++q) t[q] = kmax(t[q], t[q + w]);
    }
    const uint32_t tie = pk_key_tie(t[0]);
    const int r = (int)(tie >> 6), b = (int)(tie & 63u);
    ov[step * PK_THREADS + tid] = pk_key_score(t[0]);
    oi[step * PK_THREADS + tid] = i1s[r * PK_THREADS + tid] * n_sub + i2s[b * PK_THREADS + tid];
    const int nb = b + 1;
    const KT nk = nb < c1 ? pk_key((v1s[r * PK_THREADS + tid] + v2s[min(nb, C - 1) * PK_THREADS + tid]) * 0.5f,
                                   (uint32_t)((r << 6) | nb))
                          : kminv;
#pragma unroll
    for (int q = 0; q < C; ++q) kq[q] = q == r ? nk : kq[q];
  }
}

// Resident blocks per SM the register budget is sized for: 4 for lists up to 16, 2 for 32.
template <int C>
struct PkOcc {
  static constexpr int value = C <= 16 ? 4 : 2;
};

template <int HALF, int C>
__global__ void __launch_bounds__(PK_THREADS, PkOcc<C>::value) pk_kernel(PkArgs a, int c1, int kk) {
  pdl_enter();
  extern __shared__ float pk_smem[];
  const int hh = blockIdx.y % a.h, pr = blockIdx.y / a.h;  // pr: which address set of a paired launch
  const float* const zb = pr ? a.z2 : a.z;
  float* const svb = pr ? a.sv2 : a.sv;
  float* const wb = pr ? a.w2 : a.w;
  int32_t* const sib = pr ? a.si2 : a.si;
  const float* const gb = pr ? a.gate2 : a.gate;
  const int tid = threadIdx.x;
  const int n_sub = a.n_sub;
  float* kn1 = pk_smem;                    // (n_sub, HALF)
  float* kn2 = kn1 + n_sub * HALF;         // (n_sub, HALF)
  float* v1s = kn2 + n_sub * HALF;         // (C, PK_THREADS) per-thread sorted half lists
  int* i1s = reinterpret_cast<int*>(v1s + C * PK_THREADS);
  float* v2s = reinterpret_cast<float*>(i1s + C * PK_THREADS);
  int* i2s = reinterpret_cast<int*>(v2s + C * PK_THREADS);
  float* ov = reinterpret_cast<float*>(i2s + C * PK_THREADS);  // (kk, PK_THREADS) emitted scores
  int* oi = reinterpret_cast<int*>(ov + kk * PK_THREADS);       // (kk, PK_THREADS) emitted slot ids

  // F.normalize(keys, dim=-1) for this head
  for (int j = tid; j < 2 * n_sub; j += PK_THREADS) {
    const float* src = (j < n_sub ? a.keys1 + ((int64_t)hh * n_sub + j) * HALF
                                  : a.keys2 + ((int64_t)hh * n_sub + (j - n_sub)) * HALF);
    float kv[HALF];
    normalize_half<HALF>(src, kv);
    float* dst = (j < n_sub ? kn1 + j * HALF : kn2 + (j - n_sub) * HALF);
#pragma unroll
    for (int dd = 0; dd < HALF; ++dd) dst[dd] = kv[dd];
  }
  __syncthreads();

  const int64_t n = (int64_t)blockIdx.x * PK_THREADS + tid;
  if (n >= a.N) return;
  const float* zr = zb + n * a.ldz + (int64_t)hh * a.d_a;
  const bool zvec = HALF % 4 == 0 && ((reinterpret_cast<uintptr_t>(zb) & 15) | (a.ldz & 3) | (a.d_a & 3)) == 0;
  // the two halves one after the other through one register list (fewer live registers, more resident warps)
#pragma unroll 1
  for (int hf = 0; hf < 2; ++hf) {
    float zn[HALF];
    normalize_half<HALF>(zr + hf * HALF, zn, zvec);
    float* vs = hf ? v2s : v1s;
    int* is = hf ? i2s : i1s;
    bool done = false;
    if constexpr (C <= 16) {
      if (n_sub <= 32) {
        float* sc = ov + tid;  // this thread's scores (the emitted-score rows are free until the walk)
        uint32_t tf[C];
        if (half_topc_fast<HALF, C, PK_THREADS>(zn, hf ? kn2 : kn1, n_sub, sc, tf)) {
#pragma unroll
          for (int q = 0; q < C; ++q) {
            const uint32_t j = FK_MASK - (tf[q] & FK_MASK);
            vs[q * PK_THREADS + tid] = tf[q] ? sc[j * PK_THREADS] : -INFINITY;
            is[q * PK_THREADS + tid] = tf[q] ? (int)j : -1;
          }
        } else {
          KT tk[C];
          half_topc_stored<C, PK_THREADS>(sc, n_sub, tk);
#pragma unroll
          for (int q = 0; q < C; ++q) {
            vs[q * PK_THREADS + tid] = pk_key_score(tk[q]);
            is[q * PK_THREADS + tid] = (int)pk_key_tie(tk[q]);
          }
        }
        done = true;
      }
    }
    if (!done) {
      KT tk[C];
      half_topc<HALF, C>(zn, hf ? kn2 : kn1, n_sub, tk);
#pragma unroll
      for (int q = 0; q < C; ++q) {
        vs[q * PK_THREADS + tid] = pk_key_score(tk[q]);
        is[q * PK_THREADS + tid] = (int)pk_key_tie(tk[q]);
      }
    }
  }
  if (kk <= c1)
    walk_rows<C>(v1s, i1s, v2s, i2s, ov, oi, kk, n_sub, tid);
  else
    walk_keys<C>(v1s, i1s, v2s, i2s, ov, oi, c1, kk, n_sub, tid);
  // outputs and softmax(scale * score) (* gate); exp(scale * s - max) is kept in place of the score
  const int64_t dst = pk_dst(n, hh, a.h, a.T_bh, kk);
  const bool vec = (kk & 3) == 0 && ((reinterpret_cast<uintptr_t>(sib + dst) | (wb ? reinterpret_cast<uintptr_t>(wb + dst) : 0) |
                                      (svb ? reinterpret_cast<uintptr_t>(svb + dst) : 0)) & 15) == 0;
  if (svb) {
    for (int j = 0; j < kk; ++j) svb[dst + j] = ov[j * PK_THREADS + tid];
  }
  if (vec) {
    for (int j = 0; j < kk; j += 4)
      *reinterpret_cast<int4*>(sib + dst + j) = make_int4(oi[j * PK_THREADS + tid], oi[(j + 1) * PK_THREADS + tid],
                                                           oi[(j + 2) * PK_THREADS + tid], oi[(j + 3) * PK_THREADS + tid]);
  } else {
    for (int j = 0; j < kk; ++j) sib[dst + j] = oi[j * PK_THREADS + tid];
  }
  if (wb) {
    const float scale = expf(a.log_scale[hh]);
    float mx = -INFINITY, sum = 0.f;
    for (int j = 0; j < kk; ++j) mx = fmaxf(mx, ov[j * PK_THREADS + tid] * scale);
    for (int j = 0; j < kk; ++j) {
      const float e = expf(ov[j * PK_THREADS + tid] * scale - mx);
      ov[j * PK_THREADS + tid] = e;
      sum += e;
    }
    const float g = gb ? gb[n * a.ldgate + hh] : 1.f;
    auto wt = [&](int j) {
      const float wj = __fdiv_rn(ov[j * PK_THREADS + tid], sum);
      return gb ? wj * g : wj;
    };
    if (vec) {
      for (int j = 0; j < kk; j += 4)
        *reinterpret_cast<float4*>(wb + dst + j) = make_float4(wt(j), wt(j + 1), wt(j + 2), wt(j + 3));
    } else {
      for (int j = 0; j < kk; ++j) wb[dst + j] = wt(j);
    }
  }
}

template <int HALF, int C>
static cudaError_t launch_pk_tc(const PkArgs& a, int c1, int kk, cudaStream_t st) {
  const size_t emit_rows = (size_t)(2 * kk > a.n_sub ? 2 * kk : a.n_sub);  // emitted (score, id) rows; the fast
  // path first keeps a half's n_sub scores there
  const size_t smem = (size_t)2 * a.n_sub * HALF * 4 + (size_t)4 * C * PK_THREADS * 4 + emit_rows * PK_THREADS * 4;
  auto kern = pk_kernel<HALF, C>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)ceil_div(a.N, PK_THREADS), (unsigned)(a.h * (a.pairs > 1 ? 2 : 1)));
  LaunchScope scope_("pk_address", st);
  return launch_k(kern, dim3(grid), dim3(PK_THREADS), smem, st, a, c1, kk);
}

template <int HALF>
static cudaError_t launch_pk_half(const PkArgs& a, int c1, int kk, cudaStream_t st) {
  if (c1 <= 4) return launch_pk_tc<HALF, 4>(a, c1, kk, st);
  if (c1 <= 8) return launch_pk_tc<HALF, 8>(a, c1, kk, st);
  if (c1 <= 16) return launch_pk_tc<HALF, 16>(a, c1, kk, st);
  return launch_pk_tc<HALF, 32>(a, c1, kk, st);
}

// ------------------------------------------------------------------------------------ 32-bit-key variant
// The selection of pk_kernel with 32-bit keys for any n_sub <= 256, fewer registers and about half the shared
// memory, so more warps are resident.  A key is the score's order-preserving image with its low ib bits (ib: the
// bits of n_sub - 1) replaced by (2^ib - 1 - index); the replaced bits are kept, one byte per score, so the exact
// image of every selected score is restored.  Key order is the exact (score desc, index asc) order except between
// keys with equal high bits: an isolated such pair among the top C is put in exact order from the restored
// images; a run of three, or equal high bits between the C-th key and the best key left out (where the selected
// set itself may differ), sends the half through the exact 64-bit path -- rare: scores within ~2^-(23-ib) relative
// of each other.  Sub-key ids, the walk's per-row positions and the picks are bytes.
constexpr int PKF_THREADS = 128;

__device__ __forceinline__ uint32_t mono_image(float s) {
  const uint32_t b = __float_as_uint(s + 0.f);  // -0 -> +0
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float mono_score(uint32_t m) {
  return __uint_as_float((m & 0x80000000u) ? (m & 0x7FFFFFFFu) : ~m);
}

// The exact top-C of one half (64-bit keys) as (score, sub-key id) lists.  Out of line: the rare path.
template <int HALF, int C>
__device__ __noinline__ void half_lists_exact(const float* src, bool vec, const float* kn, int n_sub, float* vs,
                                              uint8_t* is, int tid) {
  float zn[HALF];
  normalize_half<HALF>(src, zn, vec);
  KT tk[C];
  half_topc<HALF, C>(zn, kn, n_sub, tk);
#pragma unroll
  for (int q = 0; q < C; ++q) {
    vs[q * PKF_THREADS + tid] = pk_key_score(tk[q]);
    is[q * PKF_THREADS + tid] = (uint8_t)pk_key_tie(tk[q]);
  }
}

// The top-C of one half with 32-bit keys as (score, sub-key id) lists; false when the exact path must redo it.
// score(j) gives sub-key j's cosine score; NSU > 0 bounds n_sub at compile time (the groups are then unrolled, so a
// score held in a register array is indexed statically).
template <int C, int NSU, typename ScoreFn>
__device__ __forceinline__ bool half_lists_fast_core(ScoreFn score, int n_sub, int ib, uint8_t* lowb, float* vs,
                                                    uint8_t* is, int tid) {
  const uint32_t mask = (1u << ib) - 1u;
  uint32_t tk[C];
  uint32_t disc = 0u;
  auto group = [&](int g0) {
    uint32_t gk[C];
#pragma unroll
    for (int q = 0; q < C; ++q) {
      const int j = g0 + q;
      uint32_t key = 0u;  // padding: below every real key (a real key is at least the image of -inf)
      if (j < n_sub) {
        float sc = score(j);
        if (sc != sc) sc = -INFINITY;
        const uint32_t m = mono_image(sc);
        lowb[j * PKF_THREADS + tid] = (uint8_t)(m & mask);
        key = (m & ~mask) | (mask - (uint32_t)j);
      }
      gk[q] = key;
    }
    // a group with at most C/4 real keys: those sorted, then the zero padding, is already sorted descending
    if (C >= 16 && n_sub - g0 <= C / 4)
      bitonic_sort_desc32_head<C, (C >= 16 ? C / 4 : 1)>(gk);
    else
      bitonic_sort_desc32<C>(gk);
    if (g0 == 0) {
#pragma unroll
      for (int q = 0; q < C; ++q) tk[q] = gk[q];
    } else {
      merge_top32<C>(tk, gk, disc);
    }
  };
  if constexpr (NSU > 0) {
#pragma unroll
    for (int g0 = 0; g0 < NSU; g0 += C)
      if (g0 < n_sub) group(g0);
  } else {
    for (int g0 = 0; g0 < n_sub; g0 += C) group(g0);
  }
  if (disc != 0u && tk[C - 1] != 0u && (disc >> ib) == (tk[C - 1] >> ib)) return false;
  uint32_t eqm = 0u;  // bit q: keys q and q + 1 share their high bits
#pragma unroll
  for (int q = 0; q + 1 < C; ++q) eqm |= (tk[q + 1] != 0u && (tk[q] >> ib) == (tk[q + 1] >> ib)) ? (1u << q) : 0u;
  if (eqm & (eqm >> 1)) return false;
  if (eqm) {
#pragma unroll
    for (int q = 0; q + 1 < C; ++q) {
      if ((eqm >> q) & 1u) {  // exact images; equal images keep the key order (index ascending)
        const uint32_t ja = mask - (tk[q] & mask), jb = mask - (tk[q + 1] & mask);
        const uint32_t ma = (tk[q] & ~mask) | lowb[ja * PKF_THREADS + tid];
        const uint32_t mb = (tk[q + 1] & ~mask) | lowb[jb * PKF_THREADS + tid];
        if (mb > ma) {
          const uint32_t t = tk[q];
          tk[q] = tk[q + 1];
          tk[q + 1] = t;
        }
      }
    }
  }
#pragma unroll
  for (int q = 0; q < C; ++q) {
    const uint32_t key = tk[q];
    const uint32_t j = mask - (key & mask);
    vs[q * PKF_THREADS + tid] = key ? mono_score((key & ~mask) | lowb[j * PKF_THREADS + tid]) : -INFINITY;
    is[q * PKF_THREADS + tid] = (uint8_t)j;
  }
  return true;
}
template <int HALF, int C>
__device__ __forceinline__ bool half_lists_fast(const float (&zn)[HALF], const float* kn, int n_sub, int ib,
                                               uint8_t* lowb, float* vs, uint8_t* is, int tid) {
  return half_lists_fast_core<C, 0>([&](int j) { return half_dot<HALF>(zn, kn + j * HALF); }, n_sub, ib, lowb, vs,
                                    is, tid);
}

// The walk of pk_fast_kernel.  Rows r >= C/2 (>= kk/2) can only ever contribute their first candidate ((r+1)(b+1)
// <= kk forces b = 0) and those candidates are sorted already (v1 descending, all with v2[0]), so the walk keeps a
// max tree over the head rows 0..C/2-1 only, plus the next unused tail row, which takes a step only when strictly
// larger (tail rows come later in flat-index order).  At step s the tree spans rows 0..min(s, C/2-1); the tail's
// first row cannot win before step C/2.  The rows' positions b_r are bytes in shared memory, each byte array laid
// out (rows, PKF_THREADS) with thread tid owning column tid, so regions that alias across phases stay private to
// their thread (a warp in its walk never touches a byte another warp's halves use).
template <int C>
struct WalkHT {
  static constexpr int H = C / 2;
  float kv[H];  // head row q's current candidate (q, b_q)
  int tail;     // tail rows taken; the next one is row H + tail
};

// Take step S's pick over NT head rows (and the tail when TAIL): (r, b) and its score; advance the state.
template <int C, int NT, bool TAIL>
__device__ __forceinline__ void walk_take(WalkHT<C>& w, const float* v1s, const float* v2s, uint8_t* brow,
                                          float v2_0, int c1, int tid, int& r, int& b, float& score) {
  constexpr int H = C / 2;
  float tv[NT];
  int tp[NT];
#pragma unroll
  for (int q = 0; q < NT; ++q) {
    tv[q] = w.kv[q];
    tp[q] = q;
  }
#pragma unroll
  for (int st = 1; st < NT; st <<= 1) {
#pragma unroll
    for (int q = 0; q + st < NT; q += 2 * st) {
      const bool hi = tv[q + st] > tv[q];  // the higher rows' candidate only when strictly larger
      tv[q] = hi ? tv[q + st] : tv[q];
      tp[q] = hi ? tp[q + st] : tp[q];
    }
  }
  if constexpr (TAIL) {  // the next tail row's first candidate, read afresh each step
    const int rr = H + w.tail;
    const float vt = rr < c1 ? (v1s[rr * PKF_THREADS + tid] + v2_0) * 0.5f : -INFINITY;
    if (vt > tv[0]) {
      r = rr;
      b = 0;
      score = vt + 0.f;  // -0 -> +0
      ++w.tail;
      return;
    }
  }
  {
    r = tp[0];
    b = brow[r * PKF_THREADS + tid];
    score = tv[0] + 0.f;
    const int nb = b + 1;  // b + 1 = c1 only after the last pick
    brow[r * PKF_THREADS + tid] = (uint8_t)nb;
    const float nk = (v1s[r * PKF_THREADS + tid] + v2s[min(nb, C - 1) * PKF_THREADS + tid]) * 0.5f;
#pragma unroll
    for (int q = 0; q < NT; ++q) w.kv[q] = q == r ? nk : w.kv[q];
  }
}

__device__ __forceinline__ int pick_slot_of(const uint8_t* i1s, const uint8_t* i2s, int r, int b, int n_sub,
                                            int tid) {
  return (int)i1s[r * PKF_THREADS + tid] * n_sub + (int)i2s[b * PKF_THREADS + tid];
}

template <int C>
__device__ __forceinline__ void walk_init(WalkHT<C>& w, const float* v1s, uint8_t* brow, float v2_0, int c1,
                                          int tid) {
  constexpr int H = C / 2;
#pragma unroll
  for (int q = 0; q < H; ++q) w.kv[q] = (v1s[q * PKF_THREADS + tid] + v2_0) * 0.5f;
  w.tail = 0;
}

// Every step unrolled, every pick in registers (lists up to 16): pick S's score in sc[S], its slot id in sl[S].
template <int C, int S>
__device__ __forceinline__ void walkr_step(WalkHT<C>& w, float (&sc)[C], int (&sl)[C], const float* v1s,
                                          const float* v2s, const uint8_t* i1s, const uint8_t* i2s, uint8_t* brow,
                                          float v2_0, int c1, int n_sub, int kk, int tid) {
  if constexpr (S < C) {
    if (S >= kk) return;
    constexpr int H = C / 2;
    constexpr int NT = S + 1 < H ? S + 1 : H;
    if constexpr (S < H) brow[S * PKF_THREADS + tid] = 0;  // head row S can first win at this step
    int r, b;
    walk_take<C, NT, (S >= H)>(w, v1s, v2s, brow, v2_0, c1, tid, r, b, sc[S]);
    sl[S] = pick_slot_of(i1s, i2s, r, b, n_sub, tid);
    walkr_step<C, S + 1>(w, sc, sl, v1s, v2s, i1s, i2s, brow, v2_0, c1, n_sub, kk, tid);
  }
}

// The head steps unrolled, the rest one rolled loop over the full head tree; picks (r, b) to shared memory.
template <int C, int S>
__device__ __forceinline__ void walkf_head(WalkHT<C>& w, const float* v1s, const float* v2s, uint8_t* brow,
                                          uint8_t* pick_r, uint8_t* pick_b, float v2_0, int c1, int kk, int tid) {
  if constexpr (S < C / 2) {
    if (S >= kk) return;
    brow[S * PKF_THREADS + tid] = 0;
    int r, b;
    float sc;
    walk_take<C, S + 1, false>(w, v1s, v2s, brow, v2_0, c1, tid, r, b, sc);
    pick_r[S * PKF_THREADS + tid] = (uint8_t)r;
    pick_b[S * PKF_THREADS + tid] = (uint8_t)b;
    walkf_head<C, S + 1>(w, v1s, v2s, brow, pick_r, pick_b, v2_0, c1, kk, tid);
  }
}
template <int C>
__device__ __forceinline__ void walkf(WalkHT<C>& w, const float* v1s, const float* v2s, uint8_t* brow,
                                     uint8_t* pick_r, uint8_t* pick_b, float v2_0, int c1, int kk, int tid) {
  walkf_head<C, 0>(w, v1s, v2s, brow, pick_r, pick_b, v2_0, c1, kk, tid);
#pragma unroll 1
  for (int s = C / 2; s < kk; ++s) {
    int r, b;
    float sc;
    walk_take<C, C / 2, true>(w, v1s, v2s, brow, v2_0, c1, tid, r, b, sc);
    pick_r[s * PKF_THREADS + tid] = (uint8_t)r;
    pick_b[s * PKF_THREADS + tid] = (uint8_t)b;
  }
}

// Resident blocks per SM the register budget is sized for.
template <int C>
struct PkfOcc {
  static constexpr int value = C <= 8 ? 8 : (C <= 16 ? 5 : 3);
};

template <int HALF, int C>
__global__ void __launch_bounds__(PKF_THREADS, PkfOcc<C>::value) pk_fast_kernel(PkArgs a, int c1, int kk, int ib) {
  pdl_enter();
  extern __shared__ __align__(16) float pkf_smem[];
  const int hh = blockIdx.y % a.h, pr = blockIdx.y / a.h;  // pr: which address set of a paired launch
  const float* const zb = pr ? a.z2 : a.z;
  float* const svb = pr ? a.sv2 : a.sv;
  float* const wb = pr ? a.w2 : a.w;
  int32_t* const sib = pr ? a.si2 : a.si;
  const float* const gb = pr ? a.gate2 : a.gate;
  const int tid = threadIdx.x;
  const int n_sub = a.n_sub;
  constexpr int P = PKF_THREADS;
  float* kn1 = pkf_smem;             // (n_sub, HALF)
  float* kn2 = kn1 + n_sub * HALF;   // (n_sub, HALF)
  float* v1s = kn2 + n_sub * HALF;   // (C, P) per-thread sorted half lists: scores
  float* v2s = v1s + C * P;
  uint8_t* i1s = reinterpret_cast<uint8_t*>(v2s + C * P);  // (C, P) sub-key ids
  uint8_t* i2s = i1s + C * P;
  uint8_t* lowb = i2s + C * P;  // (n_sub, P) a half's low image bits; after the halves: brow (C, P), the picks'
  uint8_t* brow = lowb;         // rows (kk, P) and columns (kk, P)
  uint8_t* pick_r = lowb + C * P;
  uint8_t* pick_b = pick_r + kk * P;

  // F.normalize(keys, dim=-1) for this head
  for (int j = tid; j < 2 * n_sub; j += P) {
    const float* src = (j < n_sub ? a.keys1 + ((int64_t)hh * n_sub + j) * HALF
                                  : a.keys2 + ((int64_t)hh * n_sub + (j - n_sub)) * HALF);
    float kv[HALF];
    normalize_half<HALF>(src, kv);
    float* dst = (j < n_sub ? kn1 + j * HALF : kn2 + (j - n_sub) * HALF);
#pragma unroll
    for (int dd = 0; dd < HALF; ++dd) dst[dd] = kv[dd];
  }
  __syncthreads();

  const int64_t n = (int64_t)blockIdx.x * P + tid;
  if (n >= a.N) return;
  const float* zr = zb + n * a.ldz + (int64_t)hh * a.d_a;
  const bool zvec = HALF % 4 == 0 && ((reinterpret_cast<uintptr_t>(zb) & 15) | (a.ldz & 3) | (a.d_a & 3)) == 0;
#pragma unroll 1
  for (int hf = 0; hf < 2; ++hf) {
    const float* src = zr + hf * HALF;
    float zn[HALF];
    normalize_half<HALF>(src, zn, zvec);
    float* vs = hf ? v2s : v1s;
    uint8_t* is = hf ? i2s : i1s;
    const float* kn = hf ? kn2 : kn1;
    if (!half_lists_fast<HALF, C>(zn, kn, n_sub, ib, lowb, vs, is, tid))
      half_lists_exact<HALF, C>(src, zvec, kn, n_sub, vs, is, tid);
  }
  const int64_t dst = pk_dst(n, hh, a.h, a.T_bh, kk);
  const bool vec = (kk & 3) == 0 && ((reinterpret_cast<uintptr_t>(sib + dst) | (wb ? reinterpret_cast<uintptr_t>(wb + dst) : 0) |
                                      (svb ? reinterpret_cast<uintptr_t>(svb + dst) : 0)) & 15) == 0;
  if constexpr (C <= 16) {
    // picks in registers; outputs and softmax(scale * score) (* gate) in pick order
    float sc[C];
    int sl[C];
    const float v2_0 = v2s[tid];
    WalkHT<C> w;
    walk_init<C>(w, v1s, brow, v2_0, c1, tid);
    walkr_step<C, 0>(w, sc, sl, v1s, v2s, i1s, i2s, brow, v2_0, c1, n_sub, kk, tid);
    if (vec) {
#pragma unroll
      for (int j = 0; j < C; j += 4) {
        if (j < kk) {
          *reinterpret_cast<int4*>(sib + dst + j) = make_int4(sl[j], sl[j + 1], sl[j + 2], sl[j + 3]);
          if (svb) *reinterpret_cast<float4*>(svb + dst + j) = make_float4(sc[j], sc[j + 1], sc[j + 2], sc[j + 3]);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < C; ++j) {
        if (j < kk) {
          sib[dst + j] = sl[j];
          if (svb) svb[dst + j] = sc[j];
        }
      }
    }
    if (wb) {
      const float scale = expf(a.log_scale[hh]);
      float mx = -INFINITY, sum = 0.f;
#pragma unroll
      for (int j = 0; j < C; ++j)
        if (j < kk) mx = fmaxf(mx, sc[j] * scale);
#pragma unroll
      for (int j = 0; j < C; ++j) {
        if (j < kk) {
          sc[j] = expf(sc[j] * scale - mx);
          sum += sc[j];
        }
      }
      const float g = gb ? gb[n * a.ldgate + hh] : 1.f, isum = __frcp_rn(sum);
#pragma unroll
      for (int j = 0; j < C; ++j) {
        if (j < kk) {
          const float wj = div_rn_by(sc[j], sum, isum);
          sc[j] = gb ? wj * g : wj;
        }
      }
      if (vec) {
#pragma unroll
        for (int j = 0; j < C; j += 4)
          if (j < kk) *reinterpret_cast<float4*>(wb + dst + j) = make_float4(sc[j], sc[j + 1], sc[j + 2], sc[j + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < C; ++j)
          if (j < kk) wb[dst + j] = sc[j];
      }
    }
    return;
  } else {  // picks in shared memory (bytes); a pick's score and slot come back from the lists
    {
      const float v2_0 = v2s[tid];
      WalkHT<C> w;
      walk_init<C>(w, v1s, brow, v2_0, c1, tid);
      walkf<C>(w, v1s, v2s, brow, pick_r, pick_b, v2_0, c1, kk, tid);
    }
    auto pick_score = [&](int j) {
      const int r = pick_r[j * P + tid], b = pick_b[j * P + tid];
      return (v1s[r * P + tid] + v2s[b * P + tid]) * 0.5f + 0.f;
    };
    auto pick_slot = [&](int j) {
      const int r = pick_r[j * P + tid], b = pick_b[j * P + tid];
      return (int)i1s[r * P + tid] * n_sub + (int)i2s[b * P + tid];
    };
    if (svb) {
      if (vec) {
        for (int j = 0; j < kk; j += 4)
          *reinterpret_cast<float4*>(svb + dst + j) =
              make_float4(pick_score(j), pick_score(j + 1), pick_score(j + 2), pick_score(j + 3));
      } else {
        for (int j = 0; j < kk; ++j) svb[dst + j] = pick_score(j);
      }
    }
    if (vec) {
      for (int j = 0; j < kk; j += 4)
        *reinterpret_cast<int4*>(sib + dst + j) = make_int4(pick_slot(j), pick_slot(j + 1), pick_slot(j + 2), pick_slot(j + 3));
    } else {
      for (int j = 0; j < kk; ++j) sib[dst + j] = pick_slot(j);
    }
    if (wb) {
      const float scale = expf(a.log_scale[hh]);
      float mx = -INFINITY, sum = 0.f;
      for (int j = 0; j < kk; ++j) mx = fmaxf(mx, pick_score(j) * scale);
      for (int j = 0; j < kk; ++j) sum += expf(pick_score(j) * scale - mx);
      const float g = gb ? gb[n * a.ldgate + hh] : 1.f, isum = __frcp_rn(sum);
      auto wt = [&](int j) {
        const float wj = div_rn_by(expf(pick_score(j) * scale - mx), sum, isum);
        return gb ? wj * g : wj;
      };
      if (vec) {
        for (int j = 0; j < kk; j += 4)
          *reinterpret_cast<float4*>(wb + dst + j) = make_float4(wt(j), wt(j + 1), wt(j + 2), wt(j + 3));
      } else {
        for (int j = 0; j < kk; ++j) wb[dst + j] = wt(j);
      }
    }
  }
}

// ------------------------------------------------------------------------------ scores on the tensor cores
// pk_tc_kernel: the RunTimeSdm addressing (address width 32, n_sub <= 32, c1 <= 16) with the cosine scores of the
// block's 128 addresses against the head's 2 x n_sub sub-keys computed as one tcgen05 product: A (128 x 32: the two
// normalised halves of each address) times B^T (64 x 32: sub-key j of half 1 in row j over the first 16 columns,
// sub-key j of half 2 in row 32 + j over the last 16, zeros elsewhere), so D[t][j] is half 1's score of sub-key j
// and D[t][32 + j] half 2's.  Every operand value v is split into three bfloat16 parts v = p0 + p1 + p2 (each the
// rounded remainder of the previous; |v - p0 - p1 - p2| <= 2^-27 |v|) and the six products p_a q_b with a + b <= 2
// are accumulated in float32, smallest first: a score's error is a few units of 2^-25, below the float32 rounding
// of the CUDA-core dot product it replaces.  The accumulator (128 lanes x 64 columns) lands in TMEM; each thread
// reads its own row (its address's 64 scores) and the selection proceeds as in pk_fast_kernel.  A half whose
// 32-bit keys cannot settle the order (rare near-ties) is re-sorted exactly (64-bit keys) from the same scores.
namespace pktc {
constexpr int NSUB = 32, NB = 2 * NSUB;
constexpr uint32_t A_PART = PKF_THREADS * 64, B_PART = NB * 64;  // rows of 32 bf16 (64 bytes), 64-byte swizzle
constexpr uint32_t OPS_BYTES = 3 * A_PART + 3 * B_PART;
constexpr uint32_t TMEM_COLS = 64;
// kind::f16: D float32, A and B bfloat16, both K-major, M = 128, N = 64
constexpr uint32_t IDESC =
    (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NB >> 3) << 17) | ((uint32_t)(PKF_THREADS >> 4) << 24);

// Shared-memory matrix descriptor, K-major, 64-byte swizzle: rows of 64 B, 8-row groups 512 B apart.
__device__ __forceinline__ uint64_t sw64_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;            // leading byte offset (unused by swizzled K-major layouts)
  d |= (uint64_t)(512 >> 4) << 32;   // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;            // descriptor version of sm_100
  d |= (uint64_t)4 << 61;            // SWIZZLE_64B
  return d;
}
__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(IDESC), "r"(accumulate));
}
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(tma::smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t pack2(bf16_t lo, bf16_t hi) {
  return (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
}
// Chunk c (values 8c .. 8c+7) of row `row` of the three parts: v (8 values) split v = p0 + p1 + p2, stored with the
// 64-byte swizzle (16-byte chunk c of row r at chunk c ^ ((r >> 1) & 3)).
__device__ __forceinline__ void put_chunk(unsigned char* base, uint32_t part_bytes, int row, int c, const float (&v)[8]) {
  uint32_t w[3][4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    bf16_t p[2][3];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const float x = v[2 * e + u];
      p[u][0] = __float2bfloat16_rn(x);
      const float r1 = x - __bfloat162float(p[u][0]);
      p[u][1] = __float2bfloat16_rn(r1);
      const float r2 = r1 - __bfloat162float(p[u][1]);
      p[u][2] = __float2bfloat16_rn(r2);
    }
#pragma unroll
    for (int q = 0; q < 3; ++q) w[q][e] = pack2(p[0][q], p[1][q]);
  }
  const uint32_t off = (uint32_t)row * 64 + ((uint32_t)(c ^ ((row >> 1) & 3)) << 4);
#pragma unroll
  for (int q = 0; q < 3; ++q)
    *reinterpret_cast<uint4*>(base + q * part_bytes + off) = make_uint4(w[q][0], w[q][1], w[q][2], w[q][3]);
}
// Row `row` of the three parts of an operand: v (32 values) split v = p0 + p1 + p2, each part's row of 64 bytes
// stored with the 64-byte swizzle (16-byte chunk c of row r at chunk c ^ ((r >> 1) & 3)).
__device__ __forceinline__ void put_row(unsigned char* base, uint32_t part_bytes, int row, const float (&v)[32]) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t w[3][4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      bf16_t p[2][3];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const float x = v[8 * c + 2 * e + u];
        p[u][0] = __float2bfloat16_rn(x);
        const float r1 = x - __bfloat162float(p[u][0]);
        p[u][1] = __float2bfloat16_rn(r1);
        const float r2 = r1 - __bfloat162float(p[u][1]);
        p[u][2] = __float2bfloat16_rn(r2);
      }
#pragma unroll
      for (int q = 0; q < 3; ++q) w[q][e] = pack2(p[0][q], p[1][q]);
    }
    const uint32_t off = (uint32_t)row * 64 + ((uint32_t)(c ^ ((row >> 1) & 3)) << 4);
#pragma unroll
    for (int q = 0; q < 3; ++q)
      *reinterpret_cast<uint4*>(base + q * part_bytes + off) = make_uint4(w[q][0], w[q][1], w[q][2], w[q][3]);
  }
}
}  // namespace pktc

// The exact top-C of one half from scores already computed (64-bit keys); the rare path of pk_tc_kernel.
template <int C, typename ScoreFn>
__device__ __forceinline__ void half_lists_exact_scores(ScoreFn score, int n_sub, float* vs, uint8_t* is, int tid) {
  KT tk[C];
#pragma unroll
  for (int g0 = 0; g0 < pktc::NSUB; g0 += C) {
    if (g0 >= n_sub) break;
    KT gk[C];
#pragma unroll
    for (int q = 0; q < C; ++q) {
      const int j = g0 + q;
      float s = -INFINITY;
      if (j < n_sub) {
        s = score(j);
        if (s != s) s = -INFINITY;
      }
      gk[q] = pk_key(s, j < n_sub ? (uint32_t)j : 0xFFFFFFFFu);
    }
    bitonic_sort_desc<C>(gk);
    if (g0 == 0) {
#pragma unroll
      for (int q = 0; q < C; ++q) tk[q] = gk[q];
    } else {
      merge_top<C>(tk, gk);
    }
  }
#pragma unroll
  for (int q = 0; q < C; ++q) {
    vs[q * PKF_THREADS + tid] = pk_key_score(tk[q]);
    is[q * PKF_THREADS + tid] = (uint8_t)pk_key_tie(tk[q]);
  }
}

template <int C>
__global__ void __launch_bounds__(PKF_THREADS, PkfOcc<C>::value) pk_tc_kernel(PkArgs a, int c1, int kk, int ib) {
  static_assert(C <= 16, "picks are kept in registers");
  pdl_enter();
  extern __shared__ __align__(1024) unsigned char pkt_raw[];
  __shared__ __align__(8) uint64_t mma_bar;
  __shared__ uint32_t tmem_slot;
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(pkt_raw) + 1023) & ~(uintptr_t)1023);
  unsigned char* opA = base;
  unsigned char* opB = base + 3 * pktc::A_PART;
  constexpr int P = PKF_THREADS;
  constexpr int HALF = 16;
  // once the product has completed, the operands' region holds the selection lists (as in pk_fast_kernel)
  float* v1s = reinterpret_cast<float*>(base);
  float* v2s = v1s + C * P;
  uint8_t* i1s = reinterpret_cast<uint8_t*>(v2s + C * P);
  uint8_t* i2s = i1s + C * P;
  uint8_t* lowb = i2s + C * P;
  uint8_t* brow = lowb;
  const int hh = blockIdx.y % a.h, pr = blockIdx.y / a.h;  // pr: which address set of a paired launch
  const float* const zb = pr ? a.z2 : a.z;
  float* const svb = pr ? a.sv2 : a.sv;
  float* const wb = pr ? a.w2 : a.w;
  int32_t* const sib = pr ? a.si2 : a.si;
  const float* const gb = pr ? a.gate2 : a.gate;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_sub = a.n_sub;

  // this thread's address, loaded first so the loads are in flight while the block sets up its sub-keys
  const int64_t n = (int64_t)blockIdx.x * P + tid;
  const bool live = n < a.N;
  float zraw[32];
  {
    const float* zr = zb + (live ? n : 0) * a.ldz + (int64_t)hh * a.d_a;
    if (((reinterpret_cast<uintptr_t>(zb) & 15) | (a.ldz & 3) | (a.d_a & 3)) == 0) {
#pragma unroll
      for (int d4 = 0; d4 < 8; ++d4) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(zr) + d4);
        zraw[4 * d4] = v.x;
        zraw[4 * d4 + 1] = v.y;
        zraw[4 * d4 + 2] = v.z;
        zraw[4 * d4 + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int dd = 0; dd < 32; ++dd) zraw[dd] = zr[dd];
    }
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tma::smem_u32(&tmem_slot)),
                 "r"(pktc::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    tma::mbar_init(&mma_bar, 1);
    tma::mbar_init_fence();
  }
  // B row j (j < 32: half 1's sub-key j in columns 0-15; 32 + j: half 2's in columns 16-31), F.normalize(keys):
  // two threads per row, eight values each (the pair shares its sum of squares by a shuffle)
  {
    const int rowb = tid >> 1, part = tid & 1;
    const int hf = rowb >= pktc::NSUB, j = rowb - hf * pktc::NSUB;
    float kv[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) kv[e] = 0.f;
    if (j < n_sub) {
      const float* src = (hf ? a.keys2 : a.keys1) + ((int64_t)hh * n_sub + j) * HALF + 8 * part;
#pragma unroll
      for (int e = 0; e < 8; ++e) kv[e] = src[e];
    }
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(kv[e], kv[e], ss);
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    // F.normalize: v / max(||v||, 1e-12), the norm as the sum of squares' correctly rounded square root
    const float nrm = fmaxf(__fsqrt_rn(ss), 1e-12f), inv = __frcp_rn(nrm);
#pragma unroll
    for (int e = 0; e < 8; ++e) kv[e] = div_rn_by(kv[e], nrm, inv);
    pktc::put_chunk(opB, pktc::B_PART, rowb, hf * 2 + part, kv);
    const float zero[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    pktc::put_chunk(opB, pktc::B_PART, rowb, (1 - hf) * 2 + part, zero);
  }
  (void)lane;
  // A: the address, both halves normalised (F.normalize: v / max(||v||, 1e-12)); a row past N stays zero
  {
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      float ss = 0.f;
#pragma unroll
      for (int dd = 0; dd < HALF; ++dd) ss = fmaf(zraw[hf * HALF + dd], zraw[hf * HALF + dd], ss);
      const float nrm = fmaxf(__fsqrt_rn(ss), 1e-12f), inv = __frcp_rn(nrm);
#pragma unroll
      for (int dd = 0; dd < HALF; ++dd) zraw[hf * HALF + dd] = live ? div_rn_by(zraw[hf * HALF + dd], nrm, inv) : 0.f;
    }
    pktc::put_row(opA, pktc::A_PART, tid, zraw);
  }
  tma::fence_proxy_async();  // the operands written here are read by the tensor cores (async proxy)
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_slot;
  if (tid == 0) {
    const uint32_t aa = tma::smem_u32(opA), bb = tma::smem_u32(opB);
    constexpr int PA[6] = {2, 1, 0, 1, 0, 0}, PB[6] = {0, 1, 2, 0, 1, 0};  // p_a q_b, smallest products first
#pragma unroll
    for (int u = 0; u < 6; ++u)
#pragma unroll
      for (int ks = 0; ks < 2; ++ks)
        pktc::mma(tmem, pktc::sw64_desc(aa + PA[u] * pktc::A_PART + ks * 32),
                  pktc::sw64_desc(bb + PB[u] * pktc::B_PART + ks * 32), (u | ks) != 0);
    pktc::commit(&mma_bar);
  }
  const bool done = tma::mbar_wait(&mma_bar, 0u);  // bounded; a wait that gave up skips the selection
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
  const bool work = live && done;
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    uint32_t r[32];
    pktc::ld32(lane_base + 32u * hf, r);  // this address's scores of half hf (every lane: the load is collective)
    float* vs = hf ? v2s : v1s;
    uint8_t* is = hf ? i2s : i1s;
    if (work && !half_lists_fast_core<C, pktc::NSUB>([&](int j) { return __uint_as_float(r[j]); }, n_sub, ib, lowb,
                                                     vs, is, tid))
      half_lists_exact_scores<C>([&](int j) { return __uint_as_float(r[j]); }, n_sub, vs, is, tid);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(pktc::TMEM_COLS) : "memory");
  }
  if (!work) return;

  const int64_t dst = pk_dst(n, hh, a.h, a.T_bh, kk);
  const bool vec = (kk & 3) == 0 && ((reinterpret_cast<uintptr_t>(sib + dst) | (wb ? reinterpret_cast<uintptr_t>(wb + dst) : 0) |
                                      (svb ? reinterpret_cast<uintptr_t>(svb + dst) : 0)) & 15) == 0;
  float sc[C];
  int sl[C];
  const float v2_0 = v2s[tid];
  WalkHT<C> w;
  walk_init<C>(w, v1s, brow, v2_0, c1, tid);
  walkr_step<C, 0>(w, sc, sl, v1s, v2s, i1s, i2s, brow, v2_0, c1, n_sub, kk, tid);
  if (vec) {
#pragma unroll
    for (int j = 0; j < C; j += 4) {
      if (j < kk) {
        *reinterpret_cast<int4*>(sib + dst + j) = make_int4(sl[j], sl[j + 1], sl[j + 2], sl[j + 3]);
        if (svb) *reinterpret_cast<float4*>(svb + dst + j) = make_float4(sc[j], sc[j + 1], sc[j + 2], sc[j + 3]);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < C; ++j) {
      if (j < kk) {
        sib[dst + j] = sl[j];
        if (svb) svb[dst + j] = sc[j];
      }
    }
  }
  if (wb) {
    const float scale = expf(a.log_scale[hh]);
    float mx = -INFINITY, sum = 0.f;
#pragma unroll
    for (int j = 0; j < C; ++j)
      if (j < kk) mx = fmaxf(mx, sc[j] * scale);
#pragma unroll
    for (int j = 0; j < C; ++j) {
      if (j < kk) {
        sc[j] = expf(sc[j] * scale - mx);
        sum += sc[j];
      }
    }
    const float g = gb ? gb[n * a.ldgate + hh] : 1.f, isum = __frcp_rn(sum);
#pragma unroll
    for (int j = 0; j < C; ++j) {
      if (j < kk) {
        const float wj = div_rn_by(sc[j], sum, isum);
        sc[j] = gb ? wj * g : wj;
      }
    }
    if (vec) {
#pragma unroll
      for (int j = 0; j < C; j += 4)
        if (j < kk) *reinterpret_cast<float4*>(wb + dst + j) = make_float4(sc[j], sc[j + 1], sc[j + 2], sc[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < C; ++j)
        if (j < kk) wb[dst + j] = sc[j];
    }
  }
}

template <int C>
static cudaError_t launch_pk_tc(const PkArgs& a, int c1, int kk, cudaStream_t st) {
  int ib = 1;
  while ((1 << ib) < a.n_sub) ++ib;
  const size_t lists = (size_t)2 * C * PKF_THREADS * 4 + (size_t)2 * C * PKF_THREADS +
                       (size_t)(a.n_sub > C + 2 * kk ? a.n_sub : C + 2 * kk) * PKF_THREADS;
  const size_t smem = 1024 + (lists > pktc::OPS_BYTES ? lists : (size_t)pktc::OPS_BYTES);
  auto kern = pk_tc_kernel<C>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)ceil_div(a.N, PKF_THREADS), (unsigned)(a.h * (a.pairs > 1 ? 2 : 1)));
  LaunchScope scope_("pk_address", st);
  return launch_k(kern, grid, dim3(PKF_THREADS), smem, st, a, c1, kk, ib);
}

template <int HALF, int C>
static cudaError_t launch_pkf(const PkArgs& a, int c1, int kk, cudaStream_t st) {
  int ib = 1;
  while ((1 << ib) < a.n_sub) ++ib;
  const size_t low_rows = (size_t)(a.n_sub > C + 2 * kk ? a.n_sub : C + 2 * kk);
  const size_t smem = (size_t)2 * a.n_sub * HALF * 4 + (size_t)2 * C * PKF_THREADS * 4 + (size_t)2 * C * PKF_THREADS +
                      low_rows * PKF_THREADS;
  auto kern = pk_fast_kernel<HALF, C>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)ceil_div(a.N, PKF_THREADS), (unsigned)(a.h * (a.pairs > 1 ? 2 : 1)));
  LaunchScope scope_("pk_address", st);
  return launch_k(kern, grid, dim3(PKF_THREADS), smem, st, a, c1, kk, ib);
}

template <int HALF>
static cudaError_t launch_pkf_half(const PkArgs& a, int c1, int kk, cudaStream_t st) {
  if (c1 <= 4) return launch_pkf<HALF, 4>(a, c1, kk, st);
  if (c1 <= 8) return launch_pkf<HALF, 8>(a, c1, kk, st);
  if (c1 <= 16) return launch_pkf<HALF, 16>(a, c1, kk, st);
  return launch_pkf<HALF, 32>(a, c1, kk, st);
}

// ------------------------------------------------------------------------------------ warp-per-address variant
// For launches with few addresses (decode: tens of tokens), one thread's serial sort chain is the whole latency.
// Here a warp owns an address and both stages are warp-wide bitonic sorts of the same 64-bit (score, tie) keys as
// the thread kernel (so the selections and their order are identical): (1) each half's n_sub scores, lane l holding
// sub-keys l*S .. l*S+S-1 (S = 1, 2 or 4 slots per lane), give the sorted top-c1; (2) the combined candidates
// (a, b) with (a+1)(b+1) <= kk -- a superset of the top-kk, since every pair (a', b') <= (a, b) ranks before
// (a, b) -- are sorted by (combined score desc, flat index a*c1+b asc) and the first kk are the selection.
constexpr int PKW_WARPS = 4;

template <int HALF, int S>
__global__ void __launch_bounds__(PKW_WARPS * 32) pk_warp_kernel(PkArgs a, int c1, int kk) {
  pdl_enter();
  extern __shared__ float pkw_smem[];
  const int hh = blockIdx.y % a.h, pr = blockIdx.y / a.h;  // pr: which address set of a paired launch
  const float* const zb = pr ? a.z2 : a.z;
  float* const svb = pr ? a.sv2 : a.sv;
  float* const wb = pr ? a.w2 : a.w;
  int32_t* const sib = pr ? a.si2 : a.si;
  const float* const gb = pr ? a.gate2 : a.gate;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int n_sub = a.n_sub;
  float* kn1 = pkw_smem;                 // (n_sub, HALF)
  float* kn2 = kn1 + n_sub * HALF;
  float* wsm = kn2 + n_sub * HALF + warp * 4 * 32;  // per warp: v1[32], i1[32], v2[32], i2[32]
  int* cand = reinterpret_cast<int*>(pkw_smem + 2 * n_sub * HALF + PKW_WARPS * 4 * 32);  // (a << 8 | b) pairs
  int* ncand = cand + 32 * S;
  for (int j = tid; j < 2 * n_sub; j += PKW_WARPS * 32) {
    const float* src = (j < n_sub ? a.keys1 + ((int64_t)hh * n_sub + j) * HALF
                                  : a.keys2 + ((int64_t)hh * n_sub + (j - n_sub)) * HALF);
    float kv[HALF];
    normalize_half<HALF>(src, kv);
    float* dst = (j < n_sub ? kn1 + j * HALF : kn2 + (j - n_sub) * HALF);
#pragma unroll
    for (int dd = 0; dd < HALF; ++dd) dst[dd] = kv[dd];
  }
  if (warp == 0) {
    const int nc = warp_candidates(cand, c1, kk);
    if (tid == 0) *ncand = nc;
  }
  __syncthreads();
  const int64_t n = (int64_t)blockIdx.x * PKW_WARPS + warp;
  if (n >= a.N) return;
  const float* zr = zb + n * a.ldz + (int64_t)hh * a.d_a;
  const bool zvec = HALF % 4 == 0 && ((reinterpret_cast<uintptr_t>(zb) & 15) | (a.ldz & 3) | (a.d_a & 3)) == 0;
  const int64_t dst = pk_dst(n, hh, a.h, a.T_bh, kk);
  warp_address<HALF, S>(zr, zvec, kn1, kn2, n_sub, c1, kk, cand, *ncand, wsm, wb ? expf(a.log_scale[hh]) : 0.f,
                        gb ? gb + n * a.ldgate + hh : nullptr, sib + dst, wb ? wb + dst : nullptr,
                        svb ? svb + dst : nullptr);
}

template <int HALF, int S>
static cudaError_t launch_pk_warp_s(const PkArgs& a, int c1, int kk, cudaStream_t st) {
  const size_t smem = (size_t)2 * a.n_sub * HALF * 4 + (size_t)PKW_WARPS * 4 * 32 * 4 + (size_t)(32 * S + 1) * 4;
  auto kern = pk_warp_kernel<HALF, S>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)ceil_div(a.N, PKW_WARPS), (unsigned)(a.h * (a.pairs > 1 ? 2 : 1)));
  LaunchScope scope_("pk_address", st);
  return launch_k(kern, dim3(grid), dim3(PKW_WARPS * 32), smem, st, a, c1, kk);
}

template <int HALF>
static cudaError_t launch_pk_warp(const PkArgs& a, int c1, int kk, cudaStream_t st) {
  switch (pk_warp_slots(a.n_sub, c1, kk)) {
    case 1: return launch_pk_warp_s<HALF, 1>(a, c1, kk, st);
    case 2: return launch_pk_warp_s<HALF, 2>(a, c1, kk, st);
    case 4: return launch_pk_warp_s<HALF, 4>(a, c1, kk, st);
    default: return cudaErrorInvalidValue;
  }
}

// Launches with at most this many addresses use the warp-per-address kernel (measured crossovers: with top-16
// lists the warp kernel keeps up with the block kernels to about 8,192 addresses; with top-32 lists over 72
// sub-keys it takes 47 us at 4,096 addresses against 43 us for pk_fast_kernel, and 82 us against 43 us at 8,192).
constexpr int64_t PK_WARP_MAX_ADDRESSES = 8192;
constexpr int64_t PK_WARP_MAX_ADDRESSES_C32 = 3072;

cudaError_t launch_pk_address(const PkArgs& a, cudaStream_t st) {
  if (a.N == 0) return cudaSuccess;
  const int c1 = a.k < a.n_sub ? a.k : a.n_sub;
  const int kk = a.k < c1 * c1 ? a.k : c1 * c1;
  const int64_t warp_max = c1 > 16 ? PK_WARP_MAX_ADDRESSES_C32 : PK_WARP_MAX_ADDRESSES;
  if (a.N * a.h * (a.pairs > 1 ? 2 : 1) <= warp_max && a.n_sub <= 128 && c1 <= 32 && kk <= 32) {
    switch (a.d_a / 2) {
      case 2: return launch_pk_warp<2>(a, c1, kk, st);
      case 4: return launch_pk_warp<4>(a, c1, kk, st);
      case 6: return launch_pk_warp<6>(a, c1, kk, st);
      case 8: return launch_pk_warp<8>(a, c1, kk, st);
      case 16: return launch_pk_warp<16>(a, c1, kk, st);
      case 32: return launch_pk_warp<32>(a, c1, kk, st);
      default: return cudaErrorInvalidValue;
    }
  }
  if (a.d_a == 32 && a.n_sub <= pktc::NSUB && c1 <= 16 && kk <= c1) {  // scores on the tensor cores
    if (c1 <= 4) return launch_pk_tc<4>(a, c1, kk, st);
    if (c1 <= 8) return launch_pk_tc<8>(a, c1, kk, st);
    return launch_pk_tc<16>(a, c1, kk, st);
  }
  if (a.n_sub <= 256 && c1 <= 32 && kk <= c1) {  // the 32-bit-key kernel (no row of the walk runs out)
    switch (a.d_a / 2) {
      case 2: return launch_pkf_half<2>(a, c1, kk, st);
      case 4: return launch_pkf_half<4>(a, c1, kk, st);
      case 6: return launch_pkf_half<6>(a, c1, kk, st);
      case 8: return launch_pkf_half<8>(a, c1, kk, st);
      case 16: return launch_pkf_half<16>(a, c1, kk, st);
      case 32: return launch_pkf_half<32>(a, c1, kk, st);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (a.d_a / 2) {
    case 2: return launch_pk_half<2>(a, c1, kk, st);
    case 4: return launch_pk_half<4>(a, c1, kk, st);
    case 6: return launch_pk_half<6>(a, c1, kk, st);
    case 8: return launch_pk_half<8>(a, c1, kk, st);
    case 16: return launch_pk_half<16>(a, c1, kk, st);
    case 32: return launch_pk_half<32>(a, c1, kk, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace sdm
