// Allocation-free variant of the fused quantized linear (b2_quant_linear).
//
// Some hosts cannot hand this library a workspace: code that runs where the
// process has already given every byte of device memory to another
// allocator (a framework's caching pool sized to the whole GPU), plugin
// hosts whose calling convention passes only inputs and outputs, and
// latency-critical callers for which cudaMalloc is off limits because it can
// synchronize the whole device.  For them this entry point keeps its staging
// buffer -- the per-token codes and scales the prologue writes and the GEMM
// reads -- in a fixed file-scope device array instead of a workspace.
//
// Costs and limits, stated for the user:
//   * every GPU that loads this library holds kNoAllocScratchBytes of device
//     memory for the array until the process exits;
//   * a call whose staging needs more than kNoAllocScratchBytes is rejected
//     with cudaErrorInvalidValue before anything is launched;
//   * all calls share the one array, so calls that overlap on the GPU (two
//     streams, two host threads without ordering) race on it and corrupt each
//     other's results; serialize them on one stream;
//   * nothing in the array needs to start at zero: within a call the
//     prologue writes every byte of it that the GEMM later reads, and bytes
//     left from an earlier call are never read;
//   * the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress, once per device, with that device current); make
//     that first call before any stream capture begins.
// The entry point itself calls no cudaMalloc, cudaFree or other allocating
// routine.
#include <mutex>

#include "../../include/b2_qlinear.h"
#include "b2_common.cuh"
#include "b2_internal.h"

namespace {

// 32 MiB: the staging of M x K codes (K rounded up to 16) plus M fp32 scales,
// e.g. M = 8192 tokens at K = 4096, or the 4096 x 3072 headline workload.
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;

__device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

// Device address of the scratch array on the current device (looked up once
// per device).  In host code `g_noalloc_scratch` names only a host-side
// stand-in, never a device address, so kernels must receive this pointer.
cudaError_t scratch_pointer(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" size_t b2_quant_linear_noalloc_max_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int b2_quant_linear_noalloc(int kind, const void* x, int x_dtype, int64_t M, int64_t K,
                                       int64_t ldx, int block, const void* w, int64_t ldw, int64_t N,
                                       const float* w_scale, int64_t w_scale_count,
                                       const void* bias, int bias_dtype, int epilogue, void* out,
                                       int out_dtype, int64_t ldc, void* stream) {
  if (M < 0 || K < 1) return static_cast<int>(cudaErrorInvalidValue);
  const size_t need = b2_quant_linear_workspace_bytes(M, K);
  if (need > kNoAllocScratchBytes) return static_cast<int>(cudaErrorInvalidValue);
  if (M == 0 || N == 0) {
    // Same argument checks as the workspace entry point, nothing to launch.
    return b2_quant_linear(kind, x, x_dtype, M, K, ldx, block, w, ldw, N, w_scale, w_scale_count,
                           bias, bias_dtype, epilogue, out, out_dtype, ldc, nullptr, 0, stream);
  }
  void* scratch = nullptr;
  cudaError_t e = scratch_pointer(&scratch);
  if (e != cudaSuccess) return static_cast<int>(e);
  return b2_quant_linear(kind, x, x_dtype, M, K, ldx, block, w, ldw, N, w_scale, w_scale_count,
                         bias, bias_dtype, epilogue, out, out_dtype, ldc, scratch,
                         kNoAllocScratchBytes, stream);
}
