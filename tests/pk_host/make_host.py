"""Emit a host-compilable copy of the 32-bit-key addressing kernel (sdmchat_b200/csrc/pk_address.cu, with the shared
pieces of pk_common.cuh) for the CPU test of its logic: the device qualifiers become nothing, the CUDA intrinsics
become their IEEE host equivalents, and the kernel body runs one thread at a time (phase 0: the block's sub-key
prologue; phase 1: threads [tid_begin, tid_end)).  Test infrastructure only."""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "..", "..", "sdmchat_b200", "csrc")

PRELUDE = r'''
#include <cstdint>
#include <cstring>
#include <cmath>
#include <algorithm>
#define __device__
#define __host__
#define __forceinline__ inline
#define __noinline__
using std::min; using std::max;
static inline uint32_t __float_as_uint(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float __uint_as_float(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline float __fdiv_rn(float a, float b) { return a / b; }
static inline float __fsqrt_rn(float a) { return std::sqrt(a); }
static inline float __frcp_rn(float a) { return 1.0f / a; }
// the kernels' shared-divisor quotient (common.cuh), with the host's fused multiply-add
static inline float div_rn_by(float x, float d, float inv) {
  const float q = x * inv;
  return std::fma(std::fma(-q, d, x), inv, q);
}
template <class T> static inline T __ldg(const T* p) { return *p; }
struct float4 { float x, y, z, w; };
struct int4 { int x, y, z, w; };
static inline float4 make_float4(float a, float b, float c, float d) { return {a, b, c, d}; }
static inline int4 make_int4(int a, int b, int c, int d) { return {a, b, c, d}; }
struct PkArgs {
  const float* z; int64_t ldz; const float* keys1; const float* keys2; int64_t N; int h, d_a, n_sub, k; int T_bh;
  float* sv; float* w; int32_t* si; const float* log_scale; const float* gate; int64_t ldgate;
  int pairs; const float* z2; float* sv2; float* w2; int32_t* si2; const float* gate2;
};
static bool g_force_exact = false;
namespace sdm {
'''


def cut(s, a, b):
    i = s.index(a)
    j = s.index(b, i)
    return s[:i] + s[j:]


def emit(out_path):
    pc = open(os.path.join(CSRC, "pk_common.cuh")).read()
    pc = pc[pc.index("namespace sdm {") + len("namespace sdm {"):pc.index("// Descending bitonic sort of the warp")]
    src = open(os.path.join(CSRC, "pk_address.cu")).read()
    body = src[src.index("namespace sdm {") + len("namespace sdm {"):
               src.index("template <int HALF, int C>\nstatic cudaError_t launch_pkf(")]
    # keep the helpers and the 32-bit-key kernel; drop the 64-bit-key thread kernel and its launchers, and the
    # tensor-core variant (its scores come from tcgen05; its selection is the same half_lists_fast_core and walk)
    body = cut(body, "template <int HALF, int C>\n__global__ void __launch_bounds__(PK_THREADS",
               "// ------------------------------------------------------------------------------------ 32-bit-key variant")
    body = body[:body.index("// ------------------------------------------------------------------------------ scores on the tensor "
                            "cores")]
    sig = ("__global__ void __launch_bounds__(PKF_THREADS, PkfOcc<C>::value) pk_fast_kernel(PkArgs a, int c1, int kk, "
           "int ib) {\n  pdl_enter();\n  extern __shared__ __align__(16) float pkf_smem[];")
    assert sig in body
    body = body.replace(sig, "void pk_fast_kernel(PkArgs a, int c1, int kk, int ib, float* pkf_smem, int bx, int by, "
                             "int tid_begin, int tid_end, int phase) {")
    body = body.replace("  const int tid = threadIdx.x;\n", "", 1)
    body = body.replace("blockIdx.y", "by").replace("blockIdx.x", "bx")
    body = body.replace("  // F.normalize(keys, dim=-1) for this head\n  for (int j = tid; j < 2 * n_sub; j += P) {",
                        "  if (phase == 0) {\n  for (int j = 0; j < 2 * n_sub; ++j) {", 1)
    old = """  __syncthreads();

  const int64_t n = (int64_t)bx * P + tid;
  if (n >= a.N) return;"""
    assert old in body
    body = body.replace(old, """  return; }
  for (int tid = tid_begin; tid < tid_end; ++tid) {
  const int64_t n = (int64_t)bx * P + tid;
  if (n >= a.N) continue;""", 1)
    body = body.replace("    return;\n  } else {  // picks", "    continue;\n  } else {  // picks")
    k = body.index("void pk_fast_kernel(")
    kend = body.index("\n}\n", body.index("if (wb) {", body.index("} else {  // picks", k)))
    body = body[:kend] + "\n  }\n}\n" + body[kend + 3:]
    body = body.replace("if (!half_lists_fast<HALF, C>(zn, kn, n_sub, ib, lowb, vs, is, tid))",
                        "if (g_force_exact || !half_lists_fast<HALF, C>(zn, kn, n_sub, ib, lowb, vs, is, tid))")
    assert "g_force_exact ||" in body
    open(out_path, "w").write(PRELUDE + pc + body + "\n}\n")


if __name__ == "__main__":
    emit(sys.argv[1])
