/* sdm_b200.h -- C ABI of the B200 (sm_100a) run-time sparse-distributed-memory path.
 *
 * Each entry point below replaces one method of the SDMCHAT reference's PyTorch modules on the hot path
 * (paths inside the SDMCHAT project; M = experiments/track4/sdmllm/track4_onesdm_models.py,
 * L = experiments/track4/sdmllm/track4_sdmllm_models.py, C = experiments/track4/sdmllm/track4_sdmllm24_fused_ce.py).
 *
 * Conventions
 *  - Every pointer is a device pointer owned by the caller (a torch tensor's data_ptr(), a cudaMalloc'd buffer).
 *    Host pointers are never accepted.  Nothing on these paths allocates device memory: the staged entry points
 *    that need intermediate buffers take a caller-provided workspace and have a *_workspace_size() query.
 *  - `stream` is a cudaStream_t passed as void*; all work is enqueued on it and the call returns without a
 *    device synchronisation.  Calls on different streams are independent.  Global mutable state is limited to:
 *    the per-module device flags that a bounded wait sets when it gives up (sdm_device_status reads and clears
 *    them) and the wait limit beside them (sdm_set_wait_limit_ns); the host launch counter and launch profiler;
 *    and the fixed scratch array of sdm_rt_decode_step_noalloc.
 *  - Every function returns an sdm_status.  Argument, shape and range errors are detected on the host before
 *    anything is launched and leave the outputs untouched.  SDM_ERR_CUDA reports a launch error.
 *  - Dtype codes: SDM_F32 (float32) or SDM_BF16 (bfloat16).  In SDM_BF16 mode activations (x, normalised
 *    activations, module outputs) are bfloat16 and matrices are bfloat16; products accumulate in float32; the
 *    run-time memory state is always float32.  In SDM_F32 mode everything is float32 (CUDA-core arithmetic).
 *  - Layouts are the reference's: x (B, T, d) row-major; per-token selections (B, h, T, k) as returned by
 *    RunTimeSdm.prepare (M:209-213); memory state mem (B, h, M, dh), cnt (B, h, M) as RunTimeSdm.last_state
 *    (M:257-258, 273).  Slot ids are int32 (the reference's are int64; values are identical).
 */
#ifndef SDM_B200_H
#define SDM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int sdm_status;
enum {
  SDM_OK = 0,
  SDM_ERR_ARG = 1,         /* null pointer, bad flag, misaligned pointer */
  SDM_ERR_SHAPE = 2,       /* sizes inconsistent or outside what the kernels support */
  SDM_ERR_RANGE = 3,       /* an index (token id, slot id) out of range */
  SDM_ERR_TIMEOUT = 4,     /* a bounded device-side wait gave up (the kernel returned early) */
  SDM_ERR_CUDA = 5,        /* a CUDA launch/runtime error */
  SDM_ERR_WORKSPACE = 6    /* the workspace given is smaller than the *_workspace_size() query returned */
};
enum { SDM_F32 = 0, SDM_BF16 = 1 };

/* ABI version of this header (bumped on any signature change). */
int sdm_abi_version(void);
/* Static text for a status code. */
const char* sdm_status_string(sdm_status s);
/* Number of kernels this library has launched since it was loaded (host-side counter; for launch accounting). */
int64_t sdm_kernel_launch_count(void);
/* Launch profiler: between sdm_profile_begin() and sdm_profile_end() every launch is bracketed by CUDA events on
 * its stream.  sdm_profile_end() synchronises those events and returns the number of (kernel, call-site tag)
 * groups (or -1 on a CUDA error); sdm_profile_group(i, ...) reports group i: kernel and tag names (NUL-terminated,
 * at most name_len bytes), launch count and summed device milliseconds. */
sdm_status sdm_profile_begin(void);
int sdm_profile_end(void);
sdm_status sdm_profile_group(int i, char* kernel, char* tag, int name_len, int* launches, double* total_ms);
/* Synchronises `stream`, then reports SDM_ERR_TIMEOUT if any bounded device-side wait (the tensor-core GEMM's
 * mbarrier waits and the scan's chunk-copy waits give up after about 4 s) gave up since the previous call, and
 * clears the flags. */
sdm_status sdm_device_status(void* stream);
/* Failure-handling checks (no counterpart in the reference, which has no device-side waits).
 * sdm_set_wait_limit_ns sets, on the current device, how long every bounded device-side wait polls before it gives
 * up (0 restores the default of about 4 s); it is synchronous, and a caller changes it only while no kernel of this
 * library is running.  sdm_wait_probe launches one thread that waits, through the same bounded wait the GEMM and
 * the scan use, on an mbarrier nothing arrives on and no copy completes: the wait gives up after the limit, the
 * kernel writes 2 to *done (device int; 1 would mean the wait completed) and returns, and the next
 * sdm_device_status reports SDM_ERR_TIMEOUT. */
sdm_status sdm_set_wait_limit_ns(uint64_t ns);
sdm_status sdm_wait_probe(int* done, void* stream);

/* ---------------------------------------------------------------------------------------- product-key address
 * pk_address (M:134-148).  z (N, h, d_a) float32, keys1/keys2 (h, n_sub, d_a/2) float32 ->
 * sv (N, h, kk) float32 descending, si (N, h, kk) int32 in [0, n_sub^2), kk = min(k, min(k, n_sub)^2).
 * Ties are broken lowest-index-first (the reference leaves the order of exactly equal scores to aten::topk).
 * Limits: d_a even, 2 <= d_a <= 64, 1 <= n_sub <= 128, 1 <= k <= 32. */
sdm_status sdm_pk_address(const float* z, const float* keys1, const float* keys2, int64_t N, int h, int d_a,
                          int n_sub, int k, float* sv, int32_t* si, void* stream);

/* ------------------------------------------------------------------------------------------------------ RMSNorm
 * RMSNorm.forward (L:69-71): y = (x * rsqrt(mean x^2 + eps)).to(dtype) * w.  x, w, y in `dtype`. */
sdm_status sdm_rmsnorm(const void* x, const void* w, int64_t rows, int d, float eps, int dtype, void* y,
                       void* stream);

/* --------------------------------------------------------------------------------------------------- RunTimeSdm
 * Parameters of one RunTimeSdm (M:154-185).  w_proj stacks the four input maps as nn.Linear weights, rows
 * wk (h*d_a) | wq (h*d_a) | wv (d) | wg (h), each row d wide.  `decay` is the per-head fade RunTimeSdm.decay()
 * returns (M:192-193).  onorm_w may be NULL when out_norm is 0. */
typedef struct {
  int d, heads, n_sub, d_a, k;
  int write_gate;      /* 1: gate = sigmoid(wg hx + b) scales every write weight (M:205-206) */
  int read_sum;        /* 1: read_mode "sum" (num); 0: "mean" (num / (den + read_eps)) (M:244) */
  int out_norm;        /* 1: per-head RMS out-norm with onorm_w (M:245-246) */
  float read_eps, out_norm_eps, norm_eps;
  int dtype;           /* SDM_F32 or SDM_BF16: dtype of x, out, norm_w, w_proj, wo */
  const void* norm_w;  /* (d) */
  const void* w_proj;  /* (2*h*d_a + d + h, d) */
  const float* wg_bias;/* (h) */
  const void* wo;      /* (d, d) */
  const float* keys1;  /* (h, n_sub, d_a/2) */
  const float* keys2;  /* (h, n_sub, d_a/2) */
  const float* addr_b; /* (h, d_a) */
  const float* log_scale; /* (h) */
  const float* decay;  /* (h) */
  const float* onorm_w;/* (h, dh) or NULL */
} sdm_rt_params;

/* Bytes of workspace sdm_rt_forward needs for a (B, T) call. */
size_t sdm_rt_forward_workspace_size(const sdm_rt_params* p, int B, int T);

/* RunTimeSdm.forward (M:249-274) as one call: prepare (M:195-213), the chunk loop (M:255-272), finish
 * (M:243-247).  x, out (B, T, d) in p->dtype.  reset (B, T) uint8 or NULL: 1 empties the memory before that
 * position reads (M:229-233).  add_residual: out = x + forward(x) rounded as the reference's residual add
 * (OneSdmLM.residual, M:540).  mem_out (B, h, M, dh) / cnt_out (B, h, M): the final state (last_state), or NULL.
 * Optional outputs (NULL to skip): siw, sir (B, h, T, k) int32, ww, wr (B, h, T, k) float32, gate (B, T, h),
 * values (B, T, d) float32 (the write values V of prepare, token-major), z (B, T, 2, h, d_a) float32 (the
 * write keys kz and read queries qz of prepare, M:199-200, addr_b added: the addresses pk_address scores),
 * num (B, T, h, dh) and den (B, T, h) float32 (the read before finish). */
sdm_status sdm_rt_forward(const sdm_rt_params* p, const void* x, int B, int T, const uint8_t* reset,
                          int add_residual, void* out, float* mem_out, float* cnt_out,
                          int32_t* siw, float* ww, int32_t* sir, float* wr, float* gate, float* values, float* z,
                          float* num, float* den, void* workspace, size_t workspace_bytes, void* stream);

/* The chunk loop (RunTimeSdm._chunk over all chunks of a window, M:215-241, 255-272; one call with T = L is one
 * _chunk) from prepared selections: siw, sir (B, h, T, k) int32; ww, wr (B, h, T, k) float32; V (B*T rows, row
 * stride ldv floats, head hh's dh values at column hh*dh); decay (h).  mem_in (B, h, M, dh) / cnt_in (B, h, M): the
 * state carried in (_chunk's mem, cnt), or both NULL for an empty memory.  reset (B, T) uint8 or NULL empties the
 * memory before that position reads (_chunk's seg / seg_prev: reset[t] = seg[t] != seg[t-1], seg[-1] = seg_prev).
 * num (B, T, h, dh), den (B, T, h) float32; mem_out / cnt_out (the state after the window) optional.  The state
 * stays resident in shared memory for the whole window; the workspace (16-byte aligned,
 * sdm_rt_scan_workspace_size bytes) holds the per-chunk slot lists. */
size_t sdm_rt_scan_workspace_size(int B, int T, int heads, int k);
sdm_status sdm_rt_scan(const int32_t* siw, const float* ww, const int32_t* sir, const float* wr, const float* V,
                       int64_t ldv, const float* decay, const uint8_t* reset, int B, int T, int heads, int n_sub,
                       int dh, int k, const float* mem_in, const float* cnt_in, float* num, float* den,
                       float* mem_out, float* cnt_out, void* workspace, size_t workspace_bytes, void* stream);

/* RunTimeSdm.finish (M:243-247): r = num / (den + read_eps) (read_mode "mean") or num; the per-head RMS out-norm
 * with onorm_w; out (N, d) in p->dtype = wo(r), plus x (N, d) when x is not NULL (the residual add of
 * OneSdmLM.residual, M:540).  num (N, h, dh) and den (N, h) float32, token-major as sdm_rt_scan writes them.  In
 * bf16 mode wo's float32 input is fed to the tensor cores as an exact bf16 hi + lo pair. */
size_t sdm_rt_finish_workspace_size(const sdm_rt_params* p, int64_t N);
sdm_status sdm_rt_finish(const sdm_rt_params* p, const float* num, const float* den, int64_t N, const void* x,
                         void* out, void* workspace, size_t workspace_bytes, void* stream);

/* Carried-state decode (new API; the reference has none, M:249-258): one token per stream through one
 * RunTimeSdm, the state read and then written in place.  x, out (S, d) in p->dtype (one token per stream).
 * mem (S, h, M, dh) float32, cnt (S, h, M) float32, scale (S, h) float32: the lazily-decayed state, the true state
 * being scale * (mem, cnt).  last_w (S, h, k) int32: the slots written at the previous step (used for fade 0),
 * initialise to -1.  A fresh stream starts with mem = cnt = 0, scale = 1.  reset (S) uint8 or NULL empties a
 * stream's state before it reads.  workspace per sdm_rt_decode_workspace_size. */
size_t sdm_rt_decode_workspace_size(const sdm_rt_params* p, int S);
sdm_status sdm_rt_decode_step(const sdm_rt_params* p, const void* x, int S, const uint8_t* reset,
                              int add_residual, void* out, float* mem, float* cnt, float* scale, int32_t* last_w,
                              void* workspace, size_t workspace_bytes, void* stream);

/* The same decode step for callers that cannot allocate device memory (no counterpart in the reference, which has
 * no decode API at all).  It allocates nothing and takes no workspace: its scratch is a fixed 8 MiB array inside
 * the library (sdm_rt_decode_noalloc_scratch_bytes()), held on every GPU that loads the library until exit.
 * Returns SDM_ERR_WORKSPACE when sdm_rt_decode_workspace_size(p, S) exceeds it (about 490 streams at d 768,
 * 12 heads, k 16).  A call made outside stream capture looks up the scratch's device address with the device
 * current and remembers it; a call inside a capture uses the remembered address, so the first call on a device (and
 * the first after a cudaDeviceReset) must come before any capture (else SDM_ERR_ARG).  Calls share the scratch;
 * calls that overlap on the GPU race on it. */
size_t sdm_rt_decode_noalloc_scratch_bytes(void);
sdm_status sdm_rt_decode_step_noalloc(const sdm_rt_params* p, const void* x, int S, const uint8_t* reset,
                                      int add_residual, void* out, float* mem, float* cnt, float* scale,
                                      int32_t* last_w, void* stream);

/* --------------------------------------------------------------------------------------------------- TrainedSdm
 * TrainedSdm.forward (M:448-457): q = wq RMSNorm(x); product-key top-k over n_sub^2 slots; softmax(scale *
 * score); weighted sum of the picked value rows; wo.  values (h, n_sub^2, dh) in dtype. */
typedef struct {
  int d, heads, n_sub, d_a, k;
  float norm_eps;
  int dtype;
  const void* norm_w;  /* (d) */
  const void* wq;      /* (h*d_a, d) */
  const float* keys1;  /* (h, n_sub, d_a/2) */
  const float* keys2;
  const void* values;  /* (h, n_sub^2, d/h) */
  const float* log_scale; /* (h) */
  const void* wo;      /* (d, d) */
} sdm_ts_params;

size_t sdm_ts_forward_workspace_size(const sdm_ts_params* p, int64_t N);
/* x, out (N, d); si (N, h, k) int32 and w (N, h, k) float32 (TrainedSdm.address, M:438-446) and the queries
 * q (N, h, d_a) float32 (M:439) optional.  add_residual as for sdm_rt_forward (M:547). */
sdm_status sdm_ts_forward(const sdm_ts_params* p, const void* x, int64_t N, int add_residual, void* out,
                          int32_t* si, float* w, float* q, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------------------ SwiGLU
 * SwiGLU.forward (L:96-97): down(silu(gate x) * up x); w_gate, w_up (f, d), w_down (d, f); f a multiple of 16.
 * In bf16 mode gate and up are one tensor-core GEMM against a packed (2f, d) weight whose epilogue applies
 * silu(g) * u (each factor rounded as the bf16 reference rounds), so only the product reaches memory.
 * sdm_swiglu_pack writes that packed weight (rows 32j .. 32j+15 = gate rows 16j .. 16j+15, the next 16 the same
 * up rows); pack once per weight update.
 * sdm_swiglu_forward: x, out (N, d); norm_w (d) or NULL: with it the input is RMSNorm(x) (OneSdmLM's mnorms[i],
 * M:544-545); add_residual: out = x + SwiGLU(...) rounded as the reference's residual add.
 * sdm_swiglu_block: x + SwiGLU(RMSNorm(x)) from the unpacked weights (packs into its workspace on every call). */
sdm_status sdm_swiglu_pack(const void* w_gate, const void* w_up, int d, int f, int dtype, void* w_gu, void* stream);
size_t sdm_swiglu_forward_workspace_size(int64_t N, int d, int f, int dtype);
sdm_status sdm_swiglu_forward(const void* x, const void* norm_w, const void* w_gu, const void* w_down, int64_t N,
                              int d, int f, float eps, int dtype, int add_residual, void* out, void* workspace,
                              size_t workspace_bytes, void* stream);
size_t sdm_swiglu_workspace_size(int64_t N, int d, int f, int dtype);
sdm_status sdm_swiglu_block(const void* x, const void* norm_w, const void* w_gate, const void* w_up,
                            const void* w_down, int64_t N, int d, int f, float eps, int dtype, void* out,
                            void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------------- tied logits
 * OneSdmLM.hidden + project (M:528-529, 550-555): h = RMSNorm_nf(x); logits = h @ E^T.
 * sdm_tied_logits writes logits (N, V) in dtype.  sdm_tied_ce_sum never materialises the logits: it writes
 * loss_sum[0] += sum over rows of (logsumexp(logits_row) - logits_row[target]) as float64 (the loss of
 * ce_chunked, C:69-80, summed), rows with target < 0 skipped.  sdm_tied_argmax writes argmax ids (N) int32
 * (greedy decode; lowest index on ties). */
size_t sdm_tied_head_workspace_size(int64_t N, int d, int V, int dtype);
sdm_status sdm_tied_logits(const void* x, const void* nf_w, const void* emb, int64_t N, int d, int V, float eps,
                           int dtype, void* logits, void* workspace, size_t workspace_bytes, void* stream);
sdm_status sdm_tied_ce_sum(const void* x, const void* nf_w, const void* emb, const int32_t* targets, int64_t N,
                           int d, int V, float eps, int dtype, double* loss_sum, void* workspace,
                           size_t workspace_bytes, void* stream);
sdm_status sdm_tied_argmax(const void* x, const void* nf_w, const void* emb, int64_t N, int d, int V, float eps,
                           int dtype, int32_t* ids, void* workspace, size_t workspace_bytes, void* stream);

/* OneSdmLM.project (M:528-529) of the tied head: logits (N, V) = h (N, d) @ emb (V, d)^T in dtype (no norm). */
sdm_status sdm_tied_project(const void* h, const void* emb, int64_t N, int d, int V, int dtype, void* logits,
                            void* stream);

/* Token table lookup (OneSdmLM.enfold, M:525-526): out (N, d) = emb[ids]; ids outside [0, V) -> SDM_ERR_RANGE
 * is reported through *bad (device int, set to 1) since ids live on the device; the row is then zero. */
sdm_status sdm_embed(const int32_t* ids, const void* emb, int64_t N, int d, int V, int dtype, void* out, int* bad,
                     void* stream);

/* Plain GEMM used by the modules above, exposed for tests: y (rows, n) = x (rows, kdim) @ w (n, kdim)^T in
 * float32 accumulation; x, w in dtype, y float32.  In SDM_BF16 mode this runs on the tcgen05 tensor cores. */
sdm_status sdm_gemm(const void* x, const void* w, int64_t rows, int kdim, int n, int dtype, float* y, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SDM_B200_H */
