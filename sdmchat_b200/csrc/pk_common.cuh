// Product-key addressing pieces shared by the addressing kernels (csrc/pk_address.cu) and the fused decode step
// (csrc/rt_decode.cu): the exact 64-bit selection keys, the cosine score, F.normalize of an address half, the
// output offset, and the warp-per-address selection (track4_onesdm_models.py:134-148, soft weights :203-206).
#pragma once
#include "kernels.cuh"

namespace sdm {

// (score, tie) as one 64-bit key whose unsigned order is the selection order: score descending, tie ascending.
// High word: the order-preserving bit image of the float score; low word: 0xFFFFFFFF - tie.  One 64-bit compare
// then orders both at once, exactly, and a compare-exchange is that compare plus four selects.
typedef unsigned long long KT;
__device__ __forceinline__ KT kmax(KT a, KT b) { return a > b ? a : b; }
__device__ __forceinline__ KT kmin(KT a, KT b) { return a > b ? b : a; }
__device__ __forceinline__ KT pk_key(float s, uint32_t tie) {
  const uint32_t b = __float_as_uint(s + 0.f);  // -0 -> +0: equal scores share one image
  const uint32_t m = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((KT)m << 32) | (KT)(0xFFFFFFFFu - tie);
}
__device__ __forceinline__ float pk_key_score(KT k) {
  const uint32_t m = (uint32_t)(k >> 32);
  return __uint_as_float((m & 0x80000000u) ? (m & 0x7FFFFFFFu) : ~m);
}
__device__ __forceinline__ uint32_t pk_key_tie(KT k) { return 0xFFFFFFFFu - (uint32_t)k; }

// Cosine score of a normalised half against one sub-key row kr (shared memory, 16-byte aligned when HALF is a
// multiple of 4): fmaf in dd order, the row read four floats at a time.
template <int HALF>
__device__ __forceinline__ float half_dot(const float (&zn)[HALF], const float* kr) {
  float s = 0.f;
  if constexpr (HALF % 4 == 0) {
#pragma unroll
    for (int d4 = 0; d4 < HALF / 4; ++d4) {
      const float4 kv = reinterpret_cast<const float4*>(kr)[d4];
      s = fmaf(zn[4 * d4], kv.x, s);
      s = fmaf(zn[4 * d4 + 1], kv.y, s);
      s = fmaf(zn[4 * d4 + 2], kv.z, s);
      s = fmaf(zn[4 * d4 + 3], kv.w, s);
    }
  } else {
#pragma unroll
    for (int dd = 0; dd < HALF; ++dd) s = fmaf(zn[dd], kr[dd], s);
  }
  return s;
}

// F.normalize of one half: src[0..HALF) / max(||src||, 1e-12).  vec: src is 16-byte aligned (HALF a multiple
// of 4) and is read four floats at a time.  RCP: the quotients from one reciprocal (div_rn_by), else one IEEE
// division each (fewer live registers, for register-capped kernels); both are correctly rounded.
template <int HALF, bool RCP = true>
__device__ __forceinline__ void normalize_half(const float* src, float (&zn)[HALF], bool vec = false) {
  if constexpr (HALF % 4 == 0) {
    if (vec) {
#pragma unroll
      for (int d4 = 0; d4 < HALF / 4; ++d4) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(src) + d4);
        zn[4 * d4] = v.x;
        zn[4 * d4 + 1] = v.y;
        zn[4 * d4 + 2] = v.z;
        zn[4 * d4 + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int dd = 0; dd < HALF; ++dd) zn[dd] = src[dd];
    }
  } else {
#pragma unroll
    for (int dd = 0; dd < HALF; ++dd) zn[dd] = src[dd];
  }
  float ss = 0.f;
#pragma unroll
  for (int dd = 0; dd < HALF; ++dd) ss = fmaf(zn[dd], zn[dd], ss);
  const float nrm = fmaxf(__fsqrt_rn(ss), 1e-12f);
  if constexpr (RCP) {
    const float inv = __frcp_rn(nrm);
#pragma unroll
    for (int dd = 0; dd < HALF; ++dd) zn[dd] = div_rn_by(zn[dd], nrm, inv);
  } else {
#pragma unroll
    for (int dd = 0; dd < HALF; ++dd) zn[dd] = __fdiv_rn(zn[dd], nrm);
  }
}

// First output element of address (token n, head hh): the (B, h, T_bh, kk) layout when T_bh > 0 (token
// n = b * T_bh + t), else (N, h, kk).  32-bit division whenever n fits.
__device__ __forceinline__ int64_t pk_dst(int64_t n, int hh, int h, int T_bh, int kk) {
  if (T_bh <= 0) return (n * h + hh) * kk;
  int64_t bb, t;
  if (n <= 0x7fffffff) {
    const uint32_t q = (uint32_t)n / (uint32_t)T_bh;
    bb = q;
    t = (uint32_t)n - q * (uint32_t)T_bh;
  } else {
    bb = n / T_bh;
    t = n % T_bh;
  }
  return ((bb * h + hh) * T_bh + t) * kk;
}

// Descending bitonic sort of the warp's 32*S keys, element e = lane*S + s in v[s].
template <int S>
__device__ __forceinline__ void warp_sort_desc(KT (&v)[S]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int size = 2; size <= 32 * S; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride >= S) {  // partner in another lane, same slot
        const int lm = stride / S;
#pragma unroll
        for (int q = 0; q < S; ++q) {
          const int e = lane * S + q;
          const KT o = __shfl_xor_sync(0xffffffffu, v[q], lm);
          const bool keep_max = ((lane & lm) == 0) == ((e & size) == 0);
          v[q] = keep_max ? (v[q] > o ? v[q] : o) : (v[q] > o ? o : v[q]);
        }
      } else {  // partner in this lane
#pragma unroll
        for (int q = 0; q < S; ++q) {
          const int q2 = q ^ stride;
          if (q2 > q) {
            const bool desc = ((lane * S + q) & size) == 0;
            const KT hi = v[q] > v[q2] ? v[q] : v[q2], lo = v[q] > v[q2] ? v[q2] : v[q];
            v[q] = desc ? hi : lo;
            v[q2] = desc ? lo : hi;
          }
        }
      }
    }
  }
}

// The candidate pairs (a, b) with a, b < c1 and (a + 1)(b + 1) <= kk, in (a, b) order, as a << 8 | b; a superset of
// the top-kk of the c1 x c1 combine (every pair (a', b') <= (a, b) ranks before (a, b)).  One warp (c1 <= 32):
// lane a counts its row, an exclusive scan places the rows.  Returns the count on every lane.
__device__ __forceinline__ int warp_candidates(int* cand, int c1, int kk) {
  const int lane = threadIdx.x & 31;
  const int cnt = lane < c1 ? min(c1, kk / (lane + 1)) : 0;
  int off = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, off, o);
    if (lane >= o) off += v;
  }
  const int total = __shfl_sync(0xffffffffu, off, 31);
  off -= cnt;
  for (int b = 0; b < cnt; ++b) cand[off + b] = (lane << 8) | b;
  return total;
}

// One warp selects one address (z at zr, its two halves of HALF floats) against the head's normalised sub-keys
// kn1/kn2 (n_sub x HALF each): (1) each half's n_sub scores, lane l holding sub-keys l*S .. l*S+S-1, sorted by
// 64-bit (score, index) keys give its top-c1; (2) the nc candidate pairs `cand`, sorted by (combined score desc,
// flat index a*c1+b asc); the first kk are the selection in order.  Writes element e < kk of the slot ids
// (si_out), the soft weights softmax(scale * score) [* gate] (w_out, when not null; scale = exp(log_scale)) and
// the scores (sv_out, when not null); wsm is 128 words of this warp's scratch (shared memory).
// One warp's sorted top-c1 of one address half (HALF floats at zh) against sub-keys kn (n_sub x HALF): lane l
// holds sub-keys l*S .. l*S+S-1, a warp-wide bitonic sort of 64-bit (score, index) keys orders them; element e < c1
// goes to vo[e] (score) and io[e] (sub-key id).
template <int HALF, int S>
__device__ __forceinline__ void warp_half_list(const float* zh, bool zvec, const float* kn, int n_sub, int c1,
                                               float* vo, int* io) {
  const int lane = threadIdx.x & 31;
  float zn[HALF];
  normalize_half<HALF>(zh, zn, zvec);
  KT key[S];
#pragma unroll
  for (int q = 0; q < S; ++q) {
    const int j = lane * S + q;
    key[q] = 0ull;  // padding: below every real key
    if (j < n_sub) {
      float sc = half_dot<HALF>(zn, kn + j * HALF);
      if (sc != sc) sc = -INFINITY;
      key[q] = pk_key(sc, (uint32_t)j);
    }
  }
  warp_sort_desc<S>(key);
#pragma unroll
  for (int q = 0; q < S; ++q) {
    const int e = lane * S + q;
    if (e < c1) {
      vo[e] = pk_key_score(key[q]);
      io[e] = (int)pk_key_tie(key[q]);
    }
  }
}

template <int S>
__device__ __forceinline__ void warp_combine(const float* wsm, int n_sub, int c1, int kk, const int* cand, int nc,
                                             float scale, const float* gate, int32_t* si_out, float* w_out,
                                             float* sv_out);

// warp_half_list with each lane normalising its own sub-keys (keys: the head's n_sub x HALF rows, global memory) in
// registers instead of reading a block-normalised copy, so no barrier precedes it: lane l scores sub-keys l*S ..
// l*S+S-1 (n_sub <= 32 S) with the same fmaf order as half_dot.  Element e < c1 of the sorted list goes to vo[e]
// (score) and io[e] (sub-key id).
template <int HALF, int S, bool RCP = true>
__device__ __forceinline__ void warp_half_list_own(const float* zh, bool zvec, const float* keys, int n_sub, int c1,
                                                   float* vo, int* io) {
  const int lane = threadIdx.x & 31;
  float zn[HALF];
  normalize_half<HALF, RCP>(zh, zn, zvec);
  KT key[S];
#pragma unroll
  for (int q = 0; q < S; ++q) {
    const int j = lane * S + q;
    key[q] = 0ull;  // padding: below every real key
    if (j < n_sub) {
      const float* kr = keys + j * HALF;
      float kv[HALF];
      normalize_half<HALF, RCP>(kr, kv, HALF % 4 == 0 && (reinterpret_cast<uintptr_t>(kr) & 15) == 0);
      float sc = 0.f;
#pragma unroll
      for (int dd = 0; dd < HALF; ++dd) sc = fmaf(zn[dd], kv[dd], sc);
      if (sc != sc) sc = -INFINITY;
      key[q] = pk_key(sc, (uint32_t)j);
    }
  }
  warp_sort_desc<S>(key);
#pragma unroll
  for (int q = 0; q < S; ++q) {
    const int e = lane * S + q;
    if (e < c1) {
      vo[e] = pk_key_score(key[q]);
      io[e] = (int)pk_key_tie(key[q]);
    }
  }
}

// One warp selects one address (z at zr, its two halves of HALF floats) against the head's normalised sub-keys
// kn1/kn2 (n_sub x HALF each): (1) each half's n_sub scores, sorted by 64-bit (score, index) keys, give its top-c1
// (warp_half_list); (2) the nc candidate pairs `cand`, sorted by (combined score desc, flat index a*c1+b asc); the
// first kk are the selection in order (warp_combine).  Writes element e < kk of the slot ids (si_out), the soft
// weights softmax(scale * score) [* gate] (w_out, when not null; scale = exp(log_scale)) and the scores (sv_out,
// when not null); wsm is 128 words of scratch (shared memory): v1[32], i1[32], v2[32], i2[32].  The two halves and
// the combine may also run on three warps (halves in parallel) with a barrier before the combine: the result is
// the same.
template <int HALF, int S>
__device__ __forceinline__ void warp_address(const float* zr, bool zvec, const float* kn1, const float* kn2,
                                             int n_sub, int c1, int kk, const int* cand, int nc, float* wsm,
                                             float scale, const float* gate, int32_t* si_out, float* w_out,
                                             float* sv_out) {
  warp_half_list<HALF, S>(zr, zvec, kn1, n_sub, c1, wsm, reinterpret_cast<int*>(wsm + 32));
  warp_half_list<HALF, S>(zr + HALF, zvec, kn2, n_sub, c1, wsm + 64, reinterpret_cast<int*>(wsm + 96));
  __syncwarp();
  warp_combine<S>(wsm, n_sub, c1, kk, cand, nc, scale, gate, si_out, w_out, sv_out);
}

template <int S>
__device__ __forceinline__ void warp_combine(const float* wsm, int n_sub, int c1, int kk, const int* cand, int nc,
                                             float scale, const float* gate, int32_t* si_out, float* w_out,
                                             float* sv_out) {
  const int lane = threadIdx.x & 31;
  const float* v1 = wsm;
  const int* i1 = reinterpret_cast<const int*>(wsm + 32);
  const float* v2 = wsm + 64;
  const int* i2 = reinterpret_cast<const int*>(wsm + 96);
  KT ck[S];
#pragma unroll
  for (int q = 0; q < S; ++q) {
    const int e = lane * S + q;
    ck[q] = 0ull;
    if (e < nc) {
      const int ab = cand[e], ra = ab >> 8, rb = ab & 255;
      ck[q] = pk_key((v1[ra] + v2[rb]) * 0.5f, (uint32_t)(ra * c1 + rb));
    }
  }
  warp_sort_desc<S>(ck);
  float sv[S], ex[S];
  const float mx = pk_key_score(__shfl_sync(0xffffffffu, ck[0], 0)) * scale;  // the first pick is the largest
#pragma unroll
  for (int q = 0; q < S; ++q) {
    const int e = lane * S + q;
    sv[q] = pk_key_score(ck[q]);
    ex[q] = e < kk ? expf(sv[q] * scale - mx) : 0.f;
    if (e < kk) {
      const int flat = (int)pk_key_tie(ck[q]), ra = flat / c1, rb = flat - ra * c1;
      si_out[e] = i1[ra] * n_sub + i2[rb];
      if (sv_out) sv_out[e] = sv[q];
    }
  }
  if (w_out) {
    // the sum in pick order, as the thread-per-address kernels add it
    float sum = 0.f;
    for (int j = 0; j < kk; ++j) {
      float ej = ex[0];
#pragma unroll
      for (int q = 1; q < S; ++q)
        if ((j % S) == q) ej = ex[q];
      sum += __shfl_sync(0xffffffffu, ej, j / S);
    }
    const float g = gate ? *gate : 1.f;
#pragma unroll
    for (int q = 0; q < S; ++q) {
      const int e = lane * S + q;
      if (e < kk) {
        float wj = __fdiv_rn(ex[q], sum);
        if (gate) wj = wj * g;
        w_out[e] = wj;
      }
    }
  }
}

// Lanes per warp-address slot count: enough for the n_sub scores of a half and the candidate pairs (0: too many).
__host__ __device__ inline int pk_warp_slots(int n_sub, int c1, int kk) {
  int nc = 0;
  for (int ra = 0; ra < c1; ++ra) nc += (kk / (ra + 1) < c1 ? kk / (ra + 1) : c1);
  const int need = n_sub > nc ? n_sub : nc;
  return need <= 32 ? 1 : (need <= 64 ? 2 : (need <= 128 ? 4 : 0));
}

}  // namespace sdm
