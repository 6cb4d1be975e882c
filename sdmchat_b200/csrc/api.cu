// The extern "C" entry points of libsdm_b200 (declared in include/sdm_b200.h): argument checks, workspace
// carving and the launch sequence of each module.  Nothing here allocates device memory.
#include "kernels.cuh"

using namespace sdm;

namespace sdm {
cudaError_t read_and_clear_timeout(int* flag, cudaStream_t st);
}  // namespace sdm

namespace {

// Bump allocator over a caller-provided workspace; with base == nullptr it only measures.
struct Bump {
  char* base;
  size_t off = 0;
  explicit Bump(void* b) : base(static_cast<char*>(b)) {}
  template <typename T>
  T* take(size_t n) {
    const size_t bytes = (n * sizeof(T) + 255) & ~(size_t)255;
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += bytes;
    return p;
  }
};

inline cudaStream_t S(void* st) { return static_cast<cudaStream_t>(st); }
inline sdm_status to_status(cudaError_t e) { return e == cudaSuccess ? SDM_OK : SDM_ERR_CUDA; }
#define SDM_TRY(...)                             \
  do {                                           \
    cudaError_t e__ = (__VA_ARGS__);             \
    if (e__ != cudaSuccess) return SDM_ERR_CUDA; \
  } while (0)

sdm_status check_rt(const sdm_rt_params* p) {
  if (!p) return SDM_ERR_ARG;
  if (p->dtype != SDM_F32 && p->dtype != SDM_BF16) return SDM_ERR_ARG;
  if (p->d <= 0 || p->heads <= 0 || p->d % p->heads) return SDM_ERR_SHAPE;
  const int half = p->d_a / 2;
  if (p->d_a % 2 || !(half == 2 || half == 4 || half == 6 || half == 8 || half == 16 || half == 32)) return SDM_ERR_SHAPE;
  if (p->n_sub < 1 || p->n_sub > 128 || p->k < 1 || p->k > 32) return SDM_ERR_SHAPE;
  const int dh = p->d / p->heads;
  if (dh > 1024) return SDM_ERR_SHAPE;
  if (!rt_scan_supported(p->n_sub * p->n_sub, dh, p->k)) return SDM_ERR_SHAPE;
  if (!p->norm_w || !p->w_proj || !p->wg_bias || !p->wo || !p->keys1 || !p->keys2 || !p->addr_b || !p->log_scale ||
      !p->decay)
    return SDM_ERR_ARG;
  if (p->out_norm && !p->onorm_w) return SDM_ERR_ARG;
  return SDM_OK;
}

inline int sel_k(int k, int n_sub) {
  const int c1 = k < n_sub ? k : n_sub;
  return k < c1 * c1 ? k : c1 * c1;
}

struct RtWs {
  void* hx;
  float* proj;
  int32_t *siw, *sir;
  float *ww, *wr, *num, *den;
  void* rbuf;
  unsigned char* rec;  // chunk records of the scan (forward only)
};

// B, T: the window shape of a forward (its scan needs chunk records); 0 for a decode step.
RtWs carve_rt(Bump& bp, const sdm_rt_params* p, int64_t N, bool own_sel, bool own_num, int B = 0, int T = 0) {
  const size_t es = p->dtype == SDM_BF16 ? 2 : 4;
  const int h = p->heads, d = p->d, kk = sel_k(p->k, p->n_sub);
  const int64_t C = 2LL * h * p->d_a + d + h;
  RtWs w{};
  w.hx = bp.take<char>(N * d * es);
  w.proj = bp.take<float>(N * C);
  if (own_sel) {
    w.siw = bp.take<int32_t>(N * h * kk);
    w.sir = bp.take<int32_t>(N * h * kk);
    w.ww = bp.take<float>(N * h * kk);
    w.wr = bp.take<float>(N * h * kk);
  }
  if (own_num) {
    w.num = bp.take<float>(N * d);
    w.den = bp.take<float>(N * h);
  }
  w.rbuf = bp.take<char>(N * d * es * (es == 2 ? 2 : 1));  // bf16: hi | lo halves of the float32 read
  w.rec = bp.take<unsigned char>(rt_scan_workspace_bytes(B, T, h, kk));
  return w;
}

// rmsnorm -> projection GEMM -> write and read addresses (+ soft weights, gate) for N tokens (token n = b*T + t).
template <typename T>
cudaError_t rt_prepare(const sdm_rt_params* p, const T* x, int64_t N, int T_bh, T* hx, float* proj, int32_t* siw,
                       float* ww, int32_t* sir, float* wr, cudaStream_t st, bool address = true) {
  const int h = p->heads, d = p->d;
  const int64_t C = 2LL * h * p->d_a + d + h;
  cudaError_t e = launch_rmsnorm<T>(x, static_cast<const T*>(p->norm_w), N, d, p->norm_eps, hx, st);
  if (e != cudaSuccess) return e;
  EpiProj ep{proj, C, p->addr_b, p->wg_bias, h * p->d_a, 2 * h * p->d_a + d};
  OpTag tag_("rt_proj");
  e = launch_gemm<T, EpiProj>(hx, d, static_cast<const T*>(p->w_proj), d, N, d, (int)C, ep, st);
  if (e != cudaSuccess || !address) return e;
  OpTag tag2_("rt_address");
  PkArgs pa{};
  pa.ldz = C;
  pa.keys1 = p->keys1;
  pa.keys2 = p->keys2;
  pa.N = N;
  pa.h = h;
  pa.d_a = p->d_a;
  pa.n_sub = p->n_sub;
  pa.k = p->k;
  pa.T_bh = T_bh;
  pa.log_scale = p->log_scale;
  pa.ldgate = C;
  // write addresses (keys, gated) and read addresses (queries) in one launch
  pa.z = proj;
  pa.w = ww;
  pa.si = siw;
  pa.gate = p->write_gate ? proj + 2LL * h * p->d_a + d : nullptr;
  pa.pairs = 2;
  pa.z2 = proj + (int64_t)h * p->d_a;
  pa.w2 = wr;
  pa.si2 = sir;
  pa.gate2 = nullptr;
  return launch_pk_address(pa, st);
}

template <typename T>
sdm_status rt_forward_t(const sdm_rt_params* p, const void* xv, int B, int T_, const uint8_t* reset, int add_res,
                        void* outv, float* mem_out, float* cnt_out, int32_t* siw_o, float* ww_o, int32_t* sir_o,
                        float* wr_o, float* gate_o, float* v_o, float* z_o, float* num_o, float* den_o, void* ws,
                        size_t ws_bytes, cudaStream_t st) {
  const int64_t N = (int64_t)B * T_;
  const int h = p->heads, d = p->d, dh = d / h, kk = sel_k(p->k, p->n_sub);
  const int64_t C = 2LL * h * p->d_a + d + h;
  const bool own_sel = !(siw_o && ww_o && sir_o && wr_o);
  const bool own_num = !(num_o && den_o);
  Bump meas(nullptr);
  carve_rt(meas, p, N, own_sel, own_num, B, T_);
  if (ws_bytes < meas.off || (meas.off && !ws)) return SDM_ERR_WORKSPACE;
  Bump bp(ws);
  RtWs w = carve_rt(bp, p, N, own_sel, own_num, B, T_);
  int32_t* siw = own_sel ? w.siw : siw_o;
  int32_t* sir = own_sel ? w.sir : sir_o;
  float* ww = own_sel ? w.ww : ww_o;
  float* wr = own_sel ? w.wr : wr_o;
  float* num = own_num ? w.num : num_o;
  float* den = own_num ? w.den : den_o;
  const T* x = static_cast<const T*>(xv);
  if (N == 0) return SDM_OK;
  SDM_TRY(rt_prepare<T>(p, x, N, T_, static_cast<T*>(w.hx), w.proj, siw, ww, sir, wr, st));
  if (gate_o)
    SDM_TRY(cudaMemcpy2DAsync(gate_o, h * sizeof(float), w.proj + 2LL * h * p->d_a + d, C * sizeof(float),
                              h * sizeof(float), N, cudaMemcpyDeviceToDevice, st));
  if (v_o)
    SDM_TRY(cudaMemcpy2DAsync(v_o, d * sizeof(float), w.proj + 2LL * h * p->d_a, C * sizeof(float), d * sizeof(float),
                              N, cudaMemcpyDeviceToDevice, st));
  if (z_o)
    SDM_TRY(cudaMemcpy2DAsync(z_o, 2 * h * p->d_a * sizeof(float), w.proj, C * sizeof(float),
                              2 * h * p->d_a * sizeof(float), N, cudaMemcpyDeviceToDevice, st));
  ScanArgs sa{};
  sa.siw = siw;
  sa.ww = ww;
  sa.sir = sir;
  sa.wr = wr;
  sa.V = w.proj + 2LL * h * p->d_a;
  sa.ldv = C;
  sa.decay = p->decay;
  sa.reset = reset;
  sa.B = B;
  sa.T = T_;
  sa.h = h;
  sa.M = p->n_sub * p->n_sub;
  sa.dh = dh;
  sa.k = kk;
  sa.num = num;
  sa.den = den;
  sa.mem_out = mem_out;
  sa.cnt_out = cnt_out;
  sa.rec = w.rec;
  SDM_TRY(launch_rt_scan(sa, st));
  OpTag tag_("rt_out");
  T* rbuf = static_cast<T*>(w.rbuf);
  constexpr int split = sizeof(T) == 2;  // wo's reference input is float32: feed it as bf16 hi + lo
  SDM_TRY(launch_rt_finish<T>(num, den, N, h, dh, p->read_sum, p->read_eps, p->out_norm, p->out_norm_eps, p->onorm_w,
                              rbuf, split, st));
  EpiResid<T> er{add_res ? x : nullptr, static_cast<T*>(outv), d};
  SDM_TRY(launch_gemm<T, EpiResid<T>>(rbuf, (1 + split) * d, static_cast<const T*>(p->wo), d, N, (1 + split) * d, d,
                                      er, st, d));
  return SDM_OK;
}

sdm_status check_ts(const sdm_ts_params* p) {
  if (!p) return SDM_ERR_ARG;
  if (p->dtype != SDM_F32 && p->dtype != SDM_BF16) return SDM_ERR_ARG;
  if (p->d <= 0 || p->heads <= 0 || p->d % p->heads) return SDM_ERR_SHAPE;
  const int half = p->d_a / 2;
  if (p->d_a % 2 || !(half == 2 || half == 4 || half == 6 || half == 8 || half == 16 || half == 32)) return SDM_ERR_SHAPE;
  if (p->n_sub < 1 || p->n_sub > 128 || p->k < 1 || p->k > 32) return SDM_ERR_SHAPE;
  if (!p->norm_w || !p->wq || !p->keys1 || !p->keys2 || !p->values || !p->log_scale || !p->wo) return SDM_ERR_ARG;
  return SDM_OK;
}

size_t ts_ws(const sdm_ts_params* p, int64_t N, bool own_si, void* base, void** hs, float** q, int32_t** si,
             float** w, void** rbuf) {
  Bump bp(base);
  const size_t es = p->dtype == SDM_BF16 ? 2 : 4;
  const int kk = sel_k(p->k, p->n_sub);
  *hs = bp.take<char>(N * p->d * es);
  *q = bp.take<float>(N * p->heads * p->d_a);
  *si = own_si ? bp.take<int32_t>(N * p->heads * kk) : nullptr;
  *w = bp.take<float>(N * p->heads * kk);
  *rbuf = bp.take<char>(N * p->d * es * (es == 2 ? 2 : 1));  // bf16: hi | lo halves of the float32 read
  return bp.off;
}

template <typename T>
sdm_status ts_forward_t(const sdm_ts_params* p, const void* xv, int64_t N, int add_res, void* outv, int32_t* si_o,
                        float* w_o, float* q_o, void* ws, size_t ws_bytes, cudaStream_t st) {
  void *hs, *rb;
  float *q, *w;
  int32_t* si;
  const size_t need = ts_ws(p, N, si_o == nullptr, nullptr, &hs, &q, &si, &w, &rb);
  if (ws_bytes < need || (need && !ws)) return SDM_ERR_WORKSPACE;
  ts_ws(p, N, si_o == nullptr, ws, &hs, &q, &si, &w, &rb);
  if (si_o) si = si_o;
  if (w_o) w = w_o;
  if (N == 0) return SDM_OK;
  const T* x = static_cast<const T*>(xv);
  const int h = p->heads, d = p->d, dh = d / h, kk = sel_k(p->k, p->n_sub);
  SDM_TRY(launch_rmsnorm<T>(x, static_cast<const T*>(p->norm_w), N, d, p->norm_eps, static_cast<T*>(hs), st));
  {
    OpTag tq_("ts_q");
    EpiF32 eq{q, (int64_t)h * p->d_a};
    SDM_TRY(launch_gemm<T, EpiF32>(static_cast<T*>(hs), d, static_cast<const T*>(p->wq), d, N, d, h * p->d_a, eq, st));
  }
  if (q_o)
    SDM_TRY(cudaMemcpyAsync(q_o, q, (size_t)N * h * p->d_a * sizeof(float), cudaMemcpyDeviceToDevice, st));
  OpTag tag_("ts");
  constexpr int split = sizeof(T) == 2;
  if (sizeof(T) == 2 && ts_addr_gather_ok(N, h, p->d_a, p->n_sub, p->k, dh) &&
      (reinterpret_cast<uintptr_t>(p->values) & 15) == 0) {  // decode-sized: selection and read in one launch
    SDM_TRY(launch_ts_addr_gather(q, (int64_t)h * p->d_a, p->keys1, p->keys2, p->log_scale, p->n_sub, p->k,
                                  static_cast<const bf16_t*>(p->values), N, h, dh, si, w,
                                  reinterpret_cast<bf16_t*>(rb), split, st));
    OpTag two_("ts_wo");
    EpiResid<T> er{add_res ? x : nullptr, static_cast<T*>(outv), d};
    SDM_TRY(launch_gemm<T, EpiResid<T>>(static_cast<T*>(rb), (1 + split) * d, static_cast<const T*>(p->wo), d, N,
                                        (1 + split) * d, d, er, st, d));
    return SDM_OK;
  }
  PkArgs pa{};
  pa.z = q;
  pa.ldz = (int64_t)h * p->d_a;
  pa.keys1 = p->keys1;
  pa.keys2 = p->keys2;
  pa.N = N;
  pa.h = h;
  pa.d_a = p->d_a;
  pa.n_sub = p->n_sub;
  pa.k = p->k;
  pa.T_bh = 0;
  pa.w = w;
  pa.si = si;
  pa.log_scale = p->log_scale;
  SDM_TRY(launch_pk_address(pa, st));
  SDM_TRY(launch_ts_gather<T>(si, w, static_cast<const T*>(p->values), N, h, p->n_sub * p->n_sub, dh, kk,
                              static_cast<T*>(rb), split, st));
  OpTag two_("ts_wo");
  EpiResid<T> er{add_res ? x : nullptr, static_cast<T*>(outv), d};
  SDM_TRY(launch_gemm<T, EpiResid<T>>(static_cast<T*>(rb), (1 + split) * d, static_cast<const T*>(p->wo), d, N,
                                      (1 + split) * d, d, er, st, d));
  return SDM_OK;
}

// Rows of the packed gate|up weight (2f, d): block j of 32 rows = gate rows [16j, 16j + 16) then up rows
// [16j, 16j + 16) (two strided 2-D copies).
cudaError_t swiglu_pack_rows(const void* wg, const void* wu, int d, int f, size_t es, void* wgu, cudaStream_t st) {
  const size_t blk = (size_t)16 * d * es;
  cudaError_t e = cudaMemcpy2DAsync(wgu, 2 * blk, wg, blk, blk, f / 16, cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return e;
  return cudaMemcpy2DAsync(static_cast<char*>(wgu) + blk, 2 * blk, wu, blk, blk, f / 16, cudaMemcpyDeviceToDevice, st);
}

// The fused path: bf16 on the tensor cores (d >= 16 and a multiple of 8; f a multiple of 16, which every entry
// point requires).  Its operands are 16-byte aligned: the normalised rows live in the workspace, an input without a
// norm is first copied there when it is not aligned, and a misaligned packed weight is refused.
bool swiglu_fused_shape(int dtype, int d) { return dtype == SDM_BF16 && d >= 16 && (d % 8) == 0; }

// Workspace of the SwiGLU entry points: the normalised (or aligned) rows and p = silu(gate) * up; the unfused path
// adds the (N, 2f) gate|up output.  `packed`: room for the packed weight too (sdm_swiglu_block).
size_t swiglu_ws(int64_t N, int d, int f, int dtype, bool packed, void* base, void** hm, void** pp, void** gu,
                 void** wgu) {
  Bump bp(base);
  const size_t es = dtype == SDM_BF16 ? 2 : 4;
  *hm = bp.take<char>(N * d * es);
  *pp = bp.take<char>(N * f * es);
  *gu = swiglu_fused_shape(dtype, d) ? nullptr : bp.take<char>(N * 2 * f * es);
  *wgu = packed ? bp.take<char>((size_t)2 * f * d * es) : nullptr;
  return bp.off;
}

template <typename T>
sdm_status swiglu_t(const void* xv, const void* nw, const void* wgu, const void* wd, int64_t N, int d, int f,
                    float eps, int add_res, void* outv, void* hm, void* pp, void* gu, cudaStream_t st) {
  if (N == 0) return SDM_OK;
  const T* x = static_cast<const T*>(xv);
  const int dtype = sizeof(T) == 2 ? SDM_BF16 : SDM_F32;
  OpTag tag_("swiglu");
  const T* h = x;
  if (nw) {
    SDM_TRY(launch_rmsnorm<T>(x, static_cast<const T*>(nw), N, d, eps, static_cast<T*>(hm), st));
    h = static_cast<const T*>(hm);
  }
  if (swiglu_fused_shape(dtype, d)) {
    if ((reinterpret_cast<uintptr_t>(wgu) & 15) != 0) return SDM_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(h) & 15) != 0) {
      SDM_TRY(cudaMemcpyAsync(hm, h, (size_t)N * d * sizeof(T), cudaMemcpyDeviceToDevice, st));
      h = static_cast<const T*>(hm);
    }
    if constexpr (sizeof(T) == 2) {
      OpTag tag2_("swiglu_gu");
      SDM_TRY(launch_gemm_tc<EpiSwiGLU>(h, d, static_cast<const bf16_t*>(wgu), d, N, d, 2 * f,
                                        EpiSwiGLU{static_cast<bf16_t*>(pp), f}, st, d));
    }
  } else {
    OpTag tag2_("swiglu_gu");
    SDM_TRY(launch_gemm<T, EpiStore<T>>(h, d, static_cast<const T*>(wgu), d, N, d, 2 * f,
                                        EpiStore<T>{static_cast<T*>(gu), 2 * f}, st));
    SDM_TRY(launch_swiglu_act<T>(static_cast<T*>(gu), N, f, static_cast<T*>(pp), st));
  }
  OpTag tag3_("swiglu_down");
  EpiResid<T> er{add_res ? x : nullptr, static_cast<T*>(outv), d};
  SDM_TRY(launch_gemm<T, EpiResid<T>>(static_cast<T*>(pp), f, static_cast<const T*>(wd), f, N, f, d, er, st));
  return SDM_OK;
}

constexpr int64_t HEAD_ROWS = 4096;  // rows of logits materialised at a time by the loss / argmax heads

size_t head_ws(int64_t N, int d, int V, int dtype, void* base, void** hbuf, float** lg, float2** part,
               float** tgt_logit) {
  Bump bp(base);
  const size_t es = dtype == SDM_BF16 ? 2 : 4;
  *hbuf = bp.take<char>(N * d * es);
  // the fused tensor-core head needs per-(row, column tile) partials; the CUDA-core head a block of logits rows
  const int64_t R = N < HEAD_ROWS ? N : HEAD_ROWS;
  const size_t fused = (size_t)N * ceil_div(V, TC_BN) * sizeof(float2) + 256 + (size_t)N * sizeof(float) + 256;
  const size_t chunk = (size_t)R * V * sizeof(float) + 256;
  char* rest = bp.take<char>(fused > chunk ? fused : chunk);
  *lg = reinterpret_cast<float*>(rest);
  *part = reinterpret_cast<float2*>(rest);
  *tgt_logit = rest ? reinterpret_cast<float*>(rest + (((size_t)N * ceil_div(V, TC_BN) * sizeof(float2) + 255) & ~(size_t)255))
                    : nullptr;
  return bp.off;
}

template <typename T>
sdm_status head_t(int mode, const void* xv, const void* nf_w, const void* emb, const int32_t* tgt, int64_t N, int d,
                  int V, float eps, void* logits, double* loss, int32_t* ids, void* ws, size_t ws_bytes,
                  cudaStream_t st) {
  void* hb;
  float* lg;
  float2* part;
  float* tl;
  const int dtype = sizeof(T) == 2 ? SDM_BF16 : SDM_F32;
  const size_t need = head_ws(N, d, V, dtype, nullptr, &hb, &lg, &part, &tl);
  if (ws_bytes < need || (need && !ws)) return SDM_ERR_WORKSPACE;
  head_ws(N, d, V, dtype, ws, &hb, &lg, &part, &tl);
  if (N == 0) return SDM_OK;
  const T* x = static_cast<const T*>(xv);
  T* h = static_cast<T*>(hb);
  OpTag tag_(mode == 0 ? "head_logits" : mode == 1 ? "head_ce" : "head_argmax");
  SDM_TRY(launch_rmsnorm<T>(x, static_cast<const T*>(nf_w), N, d, eps, h, st));
  const T* E = static_cast<const T*>(emb);
  if (mode == 0) {
    SDM_TRY(launch_gemm<T, EpiStore<T>>(h, d, E, d, N, d, V, EpiStore<T>{static_cast<T*>(logits), V}, st));
    return SDM_OK;
  }
  if constexpr (sizeof(T) == 2) {
    if (tc_gemm_supported(h, d, E, d, d, d)) {
      // fused head: the logits never leave the SM (per-tile logsumexp / argmax partials only)
      const int tiles_n = (int)ceil_div(V, TC_BN);
      if (mode == 1) {
        SDM_TRY(launch_gemm_tc<EpiCE>(h, d, E, d, N, d, V, EpiCE{tgt, part, tl}, st, d));
        SDM_TRY(launch_ce_combine(part, tl, tgt, N, tiles_n, loss, st));
      } else {
        SDM_TRY(launch_gemm_tc<EpiArgmax>(h, d, E, d, N, d, V, EpiArgmax{part}, st, d));
        SDM_TRY(launch_argmax_combine(part, N, tiles_n, ids, st));
      }
      return SDM_OK;
    }
  }
  for (int64_t r0 = 0; r0 < N; r0 += HEAD_ROWS) {
    const int64_t R = (N - r0) < HEAD_ROWS ? (N - r0) : HEAD_ROWS;
    SDM_TRY(launch_gemm<T, EpiF32R<T>>(h + r0 * d, d, E, d, R, d, V, EpiF32R<T>{lg, V}, st));
    if (mode == 1)
      SDM_TRY(launch_ce_rows(lg, R, V, tgt + r0, loss, st));
    else
      SDM_TRY(launch_argmax_rows(lg, R, V, ids + r0, st));
  }
  return SDM_OK;
}

}  // namespace

extern "C" {

int sdm_abi_version(void) { return 3; }

sdm_status sdm_device_status(void* stream) {
  int gemm = 0, scan = 0;
  if (read_and_clear_timeout(&gemm, S(stream)) != cudaSuccess) return SDM_ERR_CUDA;
  if (read_and_clear_scan_timeout(&scan, S(stream)) != cudaSuccess) return SDM_ERR_CUDA;
  return (gemm || scan) ? SDM_ERR_TIMEOUT : SDM_OK;
}

sdm_status sdm_set_wait_limit_ns(uint64_t ns) {
  if (set_gemm_wait_limit(ns) != cudaSuccess) return SDM_ERR_CUDA;
  if (set_scan_wait_limit(ns) != cudaSuccess) return SDM_ERR_CUDA;
  return SDM_OK;
}

sdm_status sdm_wait_probe(int* done, void* stream) {
  if (!done) return SDM_ERR_ARG;
  return to_status(launch_wait_probe(done, S(stream)));
}

const char* sdm_status_string(sdm_status s) {
  switch (s) {
    case SDM_OK: return "ok";
    case SDM_ERR_ARG: return "invalid argument (null or misaligned pointer, bad flag or dtype)";
    case SDM_ERR_SHAPE: return "unsupported or inconsistent shape";
    case SDM_ERR_RANGE: return "index out of range";
    case SDM_ERR_TIMEOUT: return "a bounded device-side wait gave up";
    case SDM_ERR_CUDA: return "CUDA launch or runtime error";
    case SDM_ERR_WORKSPACE: return "workspace smaller than the size query returned";
    default: return "unknown status";
  }
}

sdm_status sdm_pk_address(const float* z, const float* keys1, const float* keys2, int64_t N, int h, int d_a,
                          int n_sub, int k, float* sv, int32_t* si, void* stream) {
  if (!z || !keys1 || !keys2 || !si) return SDM_ERR_ARG;
  const int half = d_a / 2;
  if (N < 0 || h < 1 || d_a % 2 || !(half == 2 || half == 4 || half == 6 || half == 8 || half == 16 || half == 32))
    return SDM_ERR_SHAPE;
  if (n_sub < 1 || n_sub > 128 || k < 1 || k > 32) return SDM_ERR_SHAPE;
  PkArgs pa{};
  pa.z = z;
  pa.ldz = (int64_t)h * d_a;
  pa.keys1 = keys1;
  pa.keys2 = keys2;
  pa.N = N;
  pa.h = h;
  pa.d_a = d_a;
  pa.n_sub = n_sub;
  pa.k = k;
  pa.T_bh = 0;
  pa.sv = sv;
  pa.si = si;
  return to_status(launch_pk_address(pa, S(stream)));
}

sdm_status sdm_rmsnorm(const void* x, const void* w, int64_t rows, int d, float eps, int dtype, void* y,
                       void* stream) {
  if (!x || !w || !y) return SDM_ERR_ARG;
  if (rows < 0 || d < 1) return SDM_ERR_SHAPE;
  if (dtype == SDM_F32)
    return to_status(launch_rmsnorm<float>((const float*)x, (const float*)w, rows, d, eps, (float*)y, S(stream)));
  if (dtype == SDM_BF16)
    return to_status(launch_rmsnorm<bf16_t>((const bf16_t*)x, (const bf16_t*)w, rows, d, eps, (bf16_t*)y, S(stream)));
  return SDM_ERR_ARG;
}

size_t sdm_rt_forward_workspace_size(const sdm_rt_params* p, int B, int T) {
  if (check_rt(p) != SDM_OK || B < 0 || T < 0) return 0;
  Bump meas(nullptr);
  carve_rt(meas, p, (int64_t)B * T, true, true, B, T);
  return meas.off;
}

sdm_status sdm_rt_forward(const sdm_rt_params* p, const void* x, int B, int T, const uint8_t* reset,
                          int add_residual, void* out, float* mem_out, float* cnt_out, int32_t* siw, float* ww,
                          int32_t* sir, float* wr, float* gate, float* values, float* z, float* num, float* den,
                          void* workspace, size_t workspace_bytes, void* stream) {
  sdm_status s = check_rt(p);
  if (s != SDM_OK) return s;
  if (!x || !out) return SDM_ERR_ARG;
  if (B < 0 || T < 0) return SDM_ERR_SHAPE;
  if (p->dtype == SDM_BF16)
    return rt_forward_t<bf16_t>(p, x, B, T, reset, add_residual, out, mem_out, cnt_out, siw, ww, sir, wr, gate,
                                values, z, num, den, workspace, workspace_bytes, S(stream));
  return rt_forward_t<float>(p, x, B, T, reset, add_residual, out, mem_out, cnt_out, siw, ww, sir, wr, gate, values,
                             z, num, den, workspace, workspace_bytes, S(stream));
}

size_t sdm_rt_scan_workspace_size(int B, int T, int heads, int k) {
  if (B < 0 || T < 0 || heads < 1 || k < 1) return 0;
  return rt_scan_workspace_bytes(B, T, heads, k);
}

sdm_status sdm_rt_scan(const int32_t* siw, const float* ww, const int32_t* sir, const float* wr, const float* V,
                       int64_t ldv, const float* decay, const uint8_t* reset, int B, int T, int heads, int n_sub,
                       int dh, int k, const float* mem_in, const float* cnt_in, float* num, float* den,
                       float* mem_out, float* cnt_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!siw || !ww || !sir || !wr || !V || !decay || !num || !den) return SDM_ERR_ARG;
  if ((mem_in == nullptr) != (cnt_in == nullptr)) return SDM_ERR_ARG;
  if (B < 0 || T < 0 || heads < 1 || n_sub < 1 || dh < 1 || k < 1 || ldv < (int64_t)heads * dh) return SDM_ERR_SHAPE;
  if (!rt_scan_supported(n_sub * n_sub, dh, k)) return SDM_ERR_SHAPE;
  const size_t need = rt_scan_workspace_bytes(B, T, heads, k);
  if (workspace_bytes < need || (need && !workspace)) return SDM_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 15) != 0) return SDM_ERR_ARG;
  ScanArgs sa{};
  sa.siw = siw;
  sa.ww = ww;
  sa.sir = sir;
  sa.wr = wr;
  sa.V = V;
  sa.ldv = ldv;
  sa.decay = decay;
  sa.reset = reset;
  sa.B = B;
  sa.T = T;
  sa.h = heads;
  sa.M = n_sub * n_sub;
  sa.dh = dh;
  sa.k = k;
  sa.num = num;
  sa.den = den;
  sa.mem_out = mem_out;
  sa.cnt_out = cnt_out;
  sa.rec = static_cast<unsigned char*>(workspace);
  sa.mem_in = mem_in;
  sa.cnt_in = cnt_in;
  return to_status(launch_rt_scan(sa, S(stream)));
}

size_t sdm_rt_finish_workspace_size(const sdm_rt_params* p, int64_t N) {
  if (check_rt(p) != SDM_OK || N < 0) return 0;
  Bump meas(nullptr);
  meas.take<char>(N * p->d * 4);  // bf16: the read's hi | lo halves; float32: the read
  return meas.off;
}

sdm_status sdm_rt_finish(const sdm_rt_params* p, const float* num, const float* den, int64_t N, const void* x,
                         void* out, void* workspace, size_t workspace_bytes, void* stream) {
  sdm_status s = check_rt(p);
  if (s != SDM_OK) return s;
  if (!num || !den || !out) return SDM_ERR_ARG;
  if (N < 0) return SDM_ERR_SHAPE;
  const size_t need = sdm_rt_finish_workspace_size(p, N);
  if (workspace_bytes < need || (need && !workspace)) return SDM_ERR_WORKSPACE;
  if (N == 0) return SDM_OK;
  const int h = p->heads, d = p->d, dh = d / h;
  cudaStream_t st = S(stream);
  OpTag tag_("rt_out");
  if (p->dtype == SDM_BF16) {
    bf16_t* r = static_cast<bf16_t*>(workspace);
    SDM_TRY(launch_rt_finish<bf16_t>(num, den, N, h, dh, p->read_sum, p->read_eps, p->out_norm, p->out_norm_eps,
                                     p->onorm_w, r, 1, st));
    EpiResid<bf16_t> er{static_cast<const bf16_t*>(x), static_cast<bf16_t*>(out), d};
    SDM_TRY(launch_gemm<bf16_t, EpiResid<bf16_t>>(r, 2 * d, static_cast<const bf16_t*>(p->wo), d, N, 2 * d, d, er, st,
                                                  d));
  } else {
    float* r = static_cast<float*>(workspace);
    SDM_TRY(launch_rt_finish<float>(num, den, N, h, dh, p->read_sum, p->read_eps, p->out_norm, p->out_norm_eps,
                                    p->onorm_w, r, 0, st));
    EpiResid<float> er{static_cast<const float*>(x), static_cast<float*>(out), d};
    SDM_TRY(launch_gemm<float, EpiResid<float>>(r, d, static_cast<const float*>(p->wo), d, N, d, d, er, st));
  }
  return SDM_OK;
}

size_t sdm_rt_decode_workspace_size(const sdm_rt_params* p, int S_) {
  if (check_rt(p) != SDM_OK || S_ < 0) return 0;
  Bump meas(nullptr);
  carve_rt(meas, p, S_, true, true);
  return meas.off;
}

sdm_status sdm_rt_decode_step(const sdm_rt_params* p, const void* x, int S_, const uint8_t* reset, int add_residual,
                              void* out, float* mem, float* cnt, float* scale, int32_t* last_w, void* workspace,
                              size_t workspace_bytes, void* stream) {
  sdm_status s = check_rt(p);
  if (s != SDM_OK) return s;
  if (!x || !out || !mem || !cnt || !scale || !last_w) return SDM_ERR_ARG;
  if (S_ < 0) return SDM_ERR_SHAPE;
  Bump meas(nullptr);
  carve_rt(meas, p, S_, true, true);
  if (workspace_bytes < meas.off || (meas.off && !workspace)) return SDM_ERR_WORKSPACE;
  if (S_ == 0) return SDM_OK;
  Bump bp(workspace);
  RtWs w = carve_rt(bp, p, S_, true, true);
  const int h = p->heads, d = p->d, dh = d / h, kk = sel_k(p->k, p->n_sub);
  const int64_t C = 2LL * h * p->d_a + d + h;
  cudaStream_t st = S(stream);
  const bool fused = rt_decode_fused_ok(p->d_a, p->n_sub, kk);  // the step selects its slots itself
  if (p->dtype == SDM_BF16) {
    SDM_TRY(rt_prepare<bf16_t>(p, (const bf16_t*)x, S_, 1, (bf16_t*)w.hx, w.proj, w.siw, w.ww, w.sir, w.wr, st,
                               !fused));
  } else {
    SDM_TRY(rt_prepare<float>(p, (const float*)x, S_, 1, (float*)w.hx, w.proj, w.siw, w.ww, w.sir, w.wr, st,
                              !fused));
  }
  OpTag tag_("rt_decode");
  DecodeArgs da{};
  da.siw = w.siw;
  da.ww = w.ww;
  da.sir = w.sir;
  da.wr = w.wr;
  da.V = w.proj + 2LL * h * p->d_a;
  da.ldv = C;
  da.decay = p->decay;
  da.reset = reset;
  da.S = S_;
  da.h = h;
  da.M = p->n_sub * p->n_sub;
  da.dh = dh;
  da.k = kk;
  da.mem = mem;
  da.cnt = cnt;
  da.scale = scale;
  da.last_w = last_w;
  da.read_sum = p->read_sum;
  da.read_eps = p->read_eps;
  da.out_norm = p->out_norm;
  da.out_norm_eps = p->out_norm_eps;
  da.onorm_w = p->onorm_w;
  da.r = w.rbuf;
  if (fused) {
    da.proj = w.proj;
    da.ldp = C;
    da.keys1 = p->keys1;
    da.keys2 = p->keys2;
    da.log_scale = p->log_scale;
    da.n_sub = p->n_sub;
    da.d_a = p->d_a;
    da.gate_col = p->write_gate ? (int)(2LL * h * p->d_a + d) : -1;
  }
  if (p->dtype == SDM_BF16) {
    da.split = 1;
    SDM_TRY(launch_rt_decode<bf16_t>(da, st));
    EpiResid<bf16_t> er{add_residual ? (const bf16_t*)x : nullptr, (bf16_t*)out, d};
    SDM_TRY(launch_gemm<bf16_t, EpiResid<bf16_t>>((bf16_t*)w.rbuf, 2 * d, (const bf16_t*)p->wo, d, S_, 2 * d, d, er, st,
                                                  d));
  } else {
    da.split = 0;
    SDM_TRY(launch_rt_decode<float>(da, st));
    EpiResid<float> er{add_residual ? (const float*)x : nullptr, (float*)out, d};
    SDM_TRY(launch_gemm<float, EpiResid<float>>((float*)w.rbuf, d, (const float*)p->wo, d, S_, d, d, er, st));
  }
  return SDM_OK;
}

size_t sdm_ts_forward_workspace_size(const sdm_ts_params* p, int64_t N) {
  if (check_ts(p) != SDM_OK || N < 0) return 0;
  void *a, *b;
  float *q, *w;
  int32_t* si;
  return ts_ws(p, N, true, nullptr, &a, &q, &si, &w, &b);
}

sdm_status sdm_ts_forward(const sdm_ts_params* p, const void* x, int64_t N, int add_residual, void* out, int32_t* si,
                          float* w, float* q, void* workspace, size_t workspace_bytes, void* stream) {
  sdm_status s = check_ts(p);
  if (s != SDM_OK) return s;
  if (!x || !out) return SDM_ERR_ARG;
  if (N < 0) return SDM_ERR_SHAPE;
  if (p->dtype == SDM_BF16)
    return ts_forward_t<bf16_t>(p, x, N, add_residual, out, si, w, q, workspace, workspace_bytes, S(stream));
  return ts_forward_t<float>(p, x, N, add_residual, out, si, w, q, workspace, workspace_bytes, S(stream));
}

sdm_status sdm_swiglu_pack(const void* w_gate, const void* w_up, int d, int f, int dtype, void* w_gu, void* stream) {
  if (!w_gate || !w_up || !w_gu) return SDM_ERR_ARG;
  if (dtype != SDM_F32 && dtype != SDM_BF16) return SDM_ERR_ARG;
  if (d < 1 || f < 16 || f % 16) return SDM_ERR_SHAPE;
  return to_status(swiglu_pack_rows(w_gate, w_up, d, f, dtype == SDM_BF16 ? 2 : 4, w_gu, S(stream)));
}

size_t sdm_swiglu_forward_workspace_size(int64_t N, int d, int f, int dtype) {
  void *a, *b, *c, *e;
  if (N < 0 || d < 1 || f < 1) return 0;
  return swiglu_ws(N, d, f, dtype, false, nullptr, &a, &b, &c, &e);
}

static sdm_status swiglu_run(const void* x, const void* norm_w, const void* w_gu, const void* w_down, int64_t N, int d,
                             int f, float eps, int dtype, int add_res, void* out, bool pack_from, const void* wg,
                             const void* wu, void* ws, size_t wsb, cudaStream_t st) {
  void *hm, *pp, *gu, *wgu;
  const size_t need = swiglu_ws(N, d, f, dtype, pack_from, nullptr, &hm, &pp, &gu, &wgu);
  if (wsb < need || (need && !ws)) return SDM_ERR_WORKSPACE;
  swiglu_ws(N, d, f, dtype, pack_from, ws, &hm, &pp, &gu, &wgu);
  if (pack_from) {
    if (N == 0) return SDM_OK;
    SDM_TRY(swiglu_pack_rows(wg, wu, d, f, dtype == SDM_BF16 ? 2 : 4, wgu, st));
    w_gu = wgu;
  }
  if (dtype == SDM_BF16)
    return swiglu_t<bf16_t>(x, norm_w, w_gu, w_down, N, d, f, eps, add_res, out, hm, pp, gu, st);
  return swiglu_t<float>(x, norm_w, w_gu, w_down, N, d, f, eps, add_res, out, hm, pp, gu, st);
}

sdm_status sdm_swiglu_forward(const void* x, const void* norm_w, const void* w_gu, const void* w_down, int64_t N,
                              int d, int f, float eps, int dtype, int add_residual, void* out, void* workspace,
                              size_t workspace_bytes, void* stream) {
  if (!x || !w_gu || !w_down || !out) return SDM_ERR_ARG;
  if (dtype != SDM_F32 && dtype != SDM_BF16) return SDM_ERR_ARG;
  if (N < 0 || d < 1 || f < 16 || f % 16) return SDM_ERR_SHAPE;
  return swiglu_run(x, norm_w, w_gu, w_down, N, d, f, eps, dtype, add_residual, out, false, nullptr, nullptr,
                    workspace, workspace_bytes, S(stream));
}

size_t sdm_swiglu_workspace_size(int64_t N, int d, int f, int dtype) {
  void *a, *b, *c, *e;
  if (N < 0 || d < 1 || f < 1) return 0;
  return swiglu_ws(N, d, f, dtype, true, nullptr, &a, &b, &c, &e);
}

sdm_status sdm_swiglu_block(const void* x, const void* norm_w, const void* w_gate, const void* w_up,
                            const void* w_down, int64_t N, int d, int f, float eps, int dtype, void* out,
                            void* workspace, size_t workspace_bytes, void* stream) {
  if (!x || !norm_w || !w_gate || !w_up || !w_down || !out) return SDM_ERR_ARG;
  if (dtype != SDM_F32 && dtype != SDM_BF16) return SDM_ERR_ARG;
  if (N < 0 || d < 1 || f < 16 || f % 16) return SDM_ERR_SHAPE;
  return swiglu_run(x, norm_w, nullptr, w_down, N, d, f, eps, dtype, 1, out, true, w_gate, w_up, workspace,
                    workspace_bytes, S(stream));
}

size_t sdm_tied_head_workspace_size(int64_t N, int d, int V, int dtype) {
  void* a;
  float *b, *t;
  float2* c;
  return head_ws(N < 0 ? 0 : N, d, V, dtype, nullptr, &a, &b, &c, &t);
}

static sdm_status head_dispatch(int mode, const void* x, const void* nf_w, const void* emb, const int32_t* tgt,
                                int64_t N, int d, int V, float eps, int dtype, void* logits, double* loss,
                                int32_t* ids, void* ws, size_t wsb, void* stream) {
  if (!x || !nf_w || !emb) return SDM_ERR_ARG;
  if (N < 0 || d < 1 || V < 1) return SDM_ERR_SHAPE;
  if (dtype == SDM_BF16)
    return head_t<bf16_t>(mode, x, nf_w, emb, tgt, N, d, V, eps, logits, loss, ids, ws, wsb, S(stream));
  if (dtype == SDM_F32)
    return head_t<float>(mode, x, nf_w, emb, tgt, N, d, V, eps, logits, loss, ids, ws, wsb, S(stream));
  return SDM_ERR_ARG;
}

sdm_status sdm_tied_logits(const void* x, const void* nf_w, const void* emb, int64_t N, int d, int V, float eps,
                           int dtype, void* logits, void* workspace, size_t workspace_bytes, void* stream) {
  if (!logits) return SDM_ERR_ARG;
  return head_dispatch(0, x, nf_w, emb, nullptr, N, d, V, eps, dtype, logits, nullptr, nullptr, workspace,
                       workspace_bytes, stream);
}

sdm_status sdm_tied_ce_sum(const void* x, const void* nf_w, const void* emb, const int32_t* targets, int64_t N, int d,
                           int V, float eps, int dtype, double* loss_sum, void* workspace, size_t workspace_bytes,
                           void* stream) {
  if (!targets || !loss_sum) return SDM_ERR_ARG;
  return head_dispatch(1, x, nf_w, emb, targets, N, d, V, eps, dtype, nullptr, loss_sum, nullptr, workspace,
                       workspace_bytes, stream);
}

sdm_status sdm_tied_argmax(const void* x, const void* nf_w, const void* emb, int64_t N, int d, int V, float eps,
                           int dtype, int32_t* ids, void* workspace, size_t workspace_bytes, void* stream) {
  if (!ids) return SDM_ERR_ARG;
  return head_dispatch(2, x, nf_w, emb, nullptr, N, d, V, eps, dtype, nullptr, nullptr, ids, workspace,
                       workspace_bytes, stream);
}

sdm_status sdm_tied_project(const void* h, const void* emb, int64_t N, int d, int V, int dtype, void* logits,
                            void* stream) {
  if (!h || !emb || !logits) return SDM_ERR_ARG;
  if (N < 0 || d < 1 || V < 1) return SDM_ERR_SHAPE;
  OpTag tag_("head_project");
  if (dtype == SDM_BF16)
    return to_status(launch_gemm<bf16_t, EpiStore<bf16_t>>((const bf16_t*)h, d, (const bf16_t*)emb, d, N, d, V,
                                                           EpiStore<bf16_t>{(bf16_t*)logits, V}, S(stream)));
  if (dtype == SDM_F32)
    return to_status(launch_gemm<float, EpiStore<float>>((const float*)h, d, (const float*)emb, d, N, d, V,
                                                         EpiStore<float>{(float*)logits, V}, S(stream)));
  return SDM_ERR_ARG;
}

sdm_status sdm_embed(const int32_t* ids, const void* emb, int64_t N, int d, int V, int dtype, void* out, int* bad,
                     void* stream) {
  if (!ids || !emb || !out) return SDM_ERR_ARG;
  if (N < 0 || d < 1 || V < 1) return SDM_ERR_SHAPE;
  if (dtype == SDM_BF16)
    return to_status(launch_embed<bf16_t>(ids, (const bf16_t*)emb, N, d, V, (bf16_t*)out, bad, S(stream)));
  if (dtype == SDM_F32)
    return to_status(launch_embed<float>(ids, (const float*)emb, N, d, V, (float*)out, bad, S(stream)));
  return SDM_ERR_ARG;
}

sdm_status sdm_gemm(const void* x, const void* w, int64_t rows, int kdim, int n, int dtype, float* y, void* stream) {
  if (!x || !w || !y) return SDM_ERR_ARG;
  if (rows < 0 || kdim < 1 || n < 1) return SDM_ERR_SHAPE;
  if (dtype == SDM_BF16)
    return to_status(launch_gemm<bf16_t, EpiF32>((const bf16_t*)x, kdim, (const bf16_t*)w, kdim, rows, kdim, n,
                                                 EpiF32{y, n}, S(stream)));
  if (dtype == SDM_F32)
    return to_status(
        launch_gemm<float, EpiF32>((const float*)x, kdim, (const float*)w, kdim, rows, kdim, n, EpiF32{y, n}, S(stream)));
  return SDM_ERR_ARG;
}

}  // extern "C"
