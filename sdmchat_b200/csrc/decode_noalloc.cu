// The carried-state decode step without any device allocation: its scratch is a fixed array in this library.
//
// Who needs this: callers that must not allocate device memory on their decode path -- a serving engine that
// owns all device memory in a fixed pool and forbids allocations inside its per-token loop, a host runtime behind
// an FFI that has no device allocator to hand the library a workspace, or a latency-critical loop where
// cudaMalloc/cudaFree would synchronise the device and stall the other streams.  sdm_rt_decode_step needs a
// caller-provided workspace; sdm_rt_decode_step_noalloc runs the same kernels on this file's static scratch.
//
// The scratch (kScratchBytes, 8 MiB) is a file-scope __device__ array: every GPU that loads the library holds it
// until the process exits.  Host code cannot use the array's name as a device address, so its address is looked
// up (cudaGetSymbolAddress, with the device current) on every call made outside stream capture and remembered per
// device; a call made while its stream is being captured uses the remembered address.  So the first call on a
// device must come before any capture, and after a cudaDeviceReset (which reloads the module and can move the
// array) the first call must again be made outside capture.  All
// calls share the one array and it keeps the last call's contents: the decode step writes every scratch byte it
// later reads, so nothing needs clearing, but two calls whose work overlaps on the GPU (different streams, or
// different host threads, on one device) race on it and must be serialised by the caller.
#include <mutex>
#include "kernels.cuh"

namespace {

constexpr size_t kScratchBytes = (size_t)8 << 20;
__device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices];
std::mutex g_scratch_mu;

// Device address of this device's copy of the scratch array: looked up afresh outside stream capture (so it follows
// a module reload after a device reset), the remembered one during capture.
sdm_status scratch_address(cudaStream_t st, void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return SDM_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return SDM_ERR_ARG;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cap) != cudaSuccess) return SDM_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (cap == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return SDM_ERR_CUDA;
    g_scratch_addr[dev] = p;
  } else if (!g_scratch_addr[dev]) {
    return SDM_ERR_ARG;  // the first call on this device was made inside a capture
  }
  *out = g_scratch_addr[dev];
  return SDM_OK;
}

}  // namespace

extern "C" size_t sdm_rt_decode_noalloc_scratch_bytes(void) { return kScratchBytes; }

extern "C" sdm_status sdm_rt_decode_step_noalloc(const sdm_rt_params* p, const void* x, int S, const uint8_t* reset,
                                                 int add_residual, void* out, float* mem, float* cnt, float* scale,
                                                 int32_t* last_w, void* stream) {
  const size_t need = sdm_rt_decode_workspace_size(p, S);
  if (need > kScratchBytes) return SDM_ERR_WORKSPACE;  // S streams need more than the fixed scratch holds
  void* ws = nullptr;
  const sdm_status st = scratch_address(static_cast<cudaStream_t>(stream), &ws);
  if (st != SDM_OK) return st;
  return sdm_rt_decode_step(p, x, S, reset, add_residual, out, mem, cnt, scale, last_w, ws, kScratchBytes, stream);
}
