// CPU check of the 32-bit-key addressing kernel's logic (test infrastructure): the kernel body, compiled as host
// code (make_host.py), runs thread by thread on seeded inputs with a zero address and a duplicated sub-key (exact
// ties).  Checks, per shape: (1) slot ids and scores equal a brute force (exact half lists, the full c1 x c1
// combine, stable order score desc / flat index asc) bit for bit; (2) the 32-bit-key path equals the forced exact
// path bit for bit (weights too); (3) every thread writes only its own bytes of shared memory (each thread runs on
// its own copy of the block's shared memory; a byte changed by two threads is a cross-thread overlap).
#include <cstdio>
#include <cstdlib>
#include <random>
#include <utility>
#include <vector>
#include PK_HOST_HEADER
using namespace sdm;

static bool g_overlap = false;

template <int HALF, int C>
static int run(int n_sub, int k, int d_a, int N, int h, unsigned seed) {
  std::mt19937 rng(seed);
  std::normal_distribution<float> nd;
  std::vector<float> z((size_t)N * h * d_a), k1(h * n_sub * HALF), k2(h * n_sub * HALF), ls(h, 0.25f);
  for (auto& v : z) v = nd(rng);
  for (auto& v : k1) v = nd(rng);
  for (auto& v : k2) v = nd(rng);
  for (int i = 0; i < h * d_a; ++i) z[7 * h * d_a + i] = 0.f;  // a zero address: every score ties
  for (int hh = 0; hh < h; ++hh)
    for (int d = 0; d < HALF; ++d) k1[(hh * n_sub + 1) * HALF + d] = k1[(hh * n_sub) * HALF + d];
  const int c1 = std::min(k, n_sub), kk = std::min(k, c1 * c1);
  int ib = 1;
  while ((1 << ib) < n_sub) ++ib;
  const size_t low_rows = (size_t)std::max(n_sub, C + 2 * kk);
  const size_t pre = (size_t)2 * n_sub * HALF * 4;
  const size_t smem = pre + (size_t)2 * C * PKF_THREADS * 4 + (size_t)2 * C * PKF_THREADS + low_rows * PKF_THREADS;
  std::vector<float> sv[2], w[2];
  std::vector<int32_t> si[2];
  for (int pass = 0; pass < 2; ++pass) {
    g_force_exact = pass == 1;
    sv[pass].assign((size_t)N * h * kk, -7.f);
    w[pass].assign((size_t)N * h * kk, -7.f);
    si[pass].assign((size_t)N * h * kk, -7);
    PkArgs a{};
    a.z = z.data(); a.ldz = h * d_a; a.keys1 = k1.data(); a.keys2 = k2.data(); a.N = N; a.h = h; a.d_a = d_a;
    a.n_sub = n_sub; a.k = k; a.T_bh = 0; a.sv = sv[pass].data(); a.w = w[pass].data(); a.si = si[pass].data();
    a.log_scale = ls.data(); a.pairs = 1;
    std::vector<unsigned char> base(smem), cp(smem), before(smem);
    std::vector<int> owner(smem);
    for (int by = 0; by < h; ++by)
      for (int bx = 0; bx < (N + PKF_THREADS - 1) / PKF_THREADS; ++bx) {
        std::fill(base.begin(), base.end(), 0xA5);
        pk_fast_kernel<HALF, C>(a, c1, kk, ib, reinterpret_cast<float*>(base.data()), bx, by, 0, 0, 0);
        std::fill(owner.begin(), owner.end(), -1);
        for (int t = 0; t < PKF_THREADS; ++t) {
          cp = base;
          std::fill(cp.begin() + pre, cp.end(), 0x5A);
          before = cp;
          pk_fast_kernel<HALF, C>(a, c1, kk, ib, reinterpret_cast<float*>(cp.data()), bx, by, t, t + 1, 1);
          for (size_t i = 0; i < smem; ++i)
            if (cp[i] != before[i]) {
              if (owner[i] >= 0 && owner[i] != t) g_overlap = true;
              owner[i] = t;
            }
        }
      }
  }
  size_t bf_bad = 0;
  for (int64_t n = 0; n < N; ++n)
    for (int hh = 0; hh < h; ++hh) {
      std::vector<std::pair<float, int>> L[2];
      for (int hf = 0; hf < 2; ++hf) {
        const float* kraw = hf ? k2.data() : k1.data();
        float zn[HALF];
        normalize_half<HALF>(z.data() + (n * h + hh) * d_a + hf * HALF, zn);
        for (int j = 0; j < n_sub; ++j) {
          float kn[HALF];
          normalize_half<HALF>(kraw + ((size_t)hh * n_sub + j) * HALF, kn);
          float sc = half_dot<HALF>(zn, kn);
          if (sc != sc) sc = -INFINITY;
          L[hf].push_back({sc + 0.f, j});
        }
        std::stable_sort(L[hf].begin(), L[hf].end(),
                         [](auto& x, auto& y) { return x.first > y.first || (x.first == y.first && x.second < y.second); });
      }
      std::vector<std::pair<float, int>> comb;
      for (int a2 = 0; a2 < c1; ++a2)
        for (int b2 = 0; b2 < c1; ++b2) comb.push_back({(L[0][a2].first + L[1][b2].first) * 0.5f + 0.f, a2 * c1 + b2});
      std::stable_sort(comb.begin(), comb.end(),
                       [](auto& x, auto& y) { return x.first > y.first || (x.first == y.first && x.second < y.second); });
      for (int e = 0; e < kk; ++e) {
        const int a2 = comb[e].second / c1, b2 = comb[e].second % c1;
        const int slot = L[0][a2].second * n_sub + L[1][b2].second;
        const size_t i = ((size_t)n * h + hh) * kk + e;
        if (si[0][i] != slot || memcmp(&sv[0][i], &comb[e].first, 4)) ++bf_bad;
      }
    }
  size_t fe_bad = 0;
  for (size_t i = 0; i < si[0].size(); ++i)
    if (si[0][i] != si[1][i] || memcmp(&sv[0][i], &sv[1][i], 4) || memcmp(&w[0][i], &w[1][i], 4)) ++fe_bad;
  printf("n_sub %d k %d d_a %d: brute force %zu, fast vs exact %zu of %zu differ; shared-memory overlap %d\n", n_sub, k,
         d_a, bf_bad, fe_bad, si[0].size(), (int)g_overlap);
  return bf_bad || fe_bad || g_overlap;
}

int main() {
  int r = 0;
  r |= run<16, 16>(32, 16, 32, 300, 3, 1);   // RunTimeSdm: lists of 16 (picks in registers)
  r |= run<16, 32>(72, 32, 32, 300, 3, 2);   // TrainedSdm: lists of 32 (picks in shared memory, rolled tail)
  r |= run<16, 32>(103, 32, 32, 200, 2, 5);  // scaled TrainedSdm, n_sub 103
  r |= run<16, 8>(16, 8, 32, 300, 3, 3);
  r |= run<6, 8>(9, 5, 12, 300, 3, 4);
  r |= run<16, 4>(32, 4, 32, 300, 3, 6);     // the 4-head, k 4 RunTimeSdm case
  return r;
}
