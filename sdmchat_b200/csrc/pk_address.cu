// Product-key addressing on CUDA cores, float32-exact (track4_onesdm_models.py:134-148, soft weights :203-206).
//
// One thread owns one (token, head) address.  The address halves are L2-normalised, scored against the head's
// normalised sub-keys (kept in shared memory), and each half's top-c1 is found with a register bitonic network
// over 64-bit keys that encode the total order (score descending, sub-key index ascending).  The c1 x c1 cartesian combine is never
// built: a frontier walk over the two sorted lists emits the top-kk combined scores in (score descending,
// flat index a*c1+b ascending) order, which is the order a stable top-k of the reference's flattened `comb`
// gives.  Only exactly equal scores can order differently from aten::topk, whose tie order is unspecified.
#include "pk_common.cuh"

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
template <int C>
__device__ __forceinline__ void bitonic_sort_desc32(uint32_t (&k)[C]) {
#pragma unroll
  for (int size = 2; size <= C; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
#pragma unroll
      for (int i = 0; i < C; ++i) {
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
template <int HALF, int C>
__device__ __forceinline__ bool half_lists_fast(const float (&zn)[HALF], const float* kn, int n_sub, int ib,
                                               uint8_t* lowb, float* vs, uint8_t* is, int tid) {
  const uint32_t mask = (1u << ib) - 1u;
  uint32_t tk[C];
  uint32_t disc = 0u;
  for (int g0 = 0; g0 < n_sub; g0 += C) {
    uint32_t gk[C];
#pragma unroll
    for (int q = 0; q < C; ++q) {
      const int j = g0 + q;
      uint32_t key = 0u;  // padding: below every real key (a real key is at least the image of -inf)
      if (j < n_sub) {
        float sc = half_dot<HALF>(zn, kn + j * HALF);
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
      const float g = gb ? gb[n * a.ldgate + hh] : 1.f;
#pragma unroll
      for (int j = 0; j < C; ++j) {
        if (j < kk) {
          const float wj = __fdiv_rn(sc[j], sum);
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
      const float g = gb ? gb[n * a.ldgate + hh] : 1.f;
      auto wt = [&](int j) {
        const float wj = __fdiv_rn(expf(pick_score(j) * scale - mx), sum);
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

// Launches with at most this many addresses use the warp-per-address kernel.
constexpr int64_t PK_WARP_MAX_ADDRESSES = 8192;

cudaError_t launch_pk_address(const PkArgs& a, cudaStream_t st) {
  if (a.N == 0) return cudaSuccess;
  const int c1 = a.k < a.n_sub ? a.k : a.n_sub;
  const int kk = a.k < c1 * c1 ? a.k : c1 * c1;
  if (a.N * a.h * (a.pairs > 1 ? 2 : 1) <= PK_WARP_MAX_ADDRESSES && a.n_sub <= 128 && c1 <= 32 && kk <= 32) {
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
