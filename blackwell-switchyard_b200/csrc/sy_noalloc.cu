// sy_noalloc.cu -- backward for callers that cannot allocate device memory.
//
// sy_bwd needs a caller-provided buffer of fp32 dw partial rows (scratch that is
// neither an input nor an output). Some callers have no way to provide one:
// code embedded in a host framework that owns every byte of device memory and
// forbids raw allocations (a plugin that may only use the tensors it is
// handed), or a latency-critical loop where an allocation -- and the device
// synchronisation cudaMalloc/cudaFree can imply -- is not acceptable.
// sy_bwd_noalloc serves them: it keeps the partial rows in a fixed-size array
// that is part of this library's device image, so the caller passes only the
// inputs and the outputs (dv and the final dw).
//
// Properties a caller must know:
//  * The array holds kNoAllocScratchFloats fp32 values (8 MiB) on every GPU
//    that loads the library, until the process exits. A shape whose partial
//    rows (sy_bwd_partials(N, BT, D, dtype) * D floats) do not fit is rejected
//    with SY_ERR_SCRATCH before anything is launched.
//  * The first call on each device looks the array's device address up
//    (cudaGetSymbolAddress, with that device current) and caches it; make that
//    first call before any stream capture.
//  * Every call on a device uses the same array. Each call overwrites every
//    partial row it later reads (nothing in it needs to start at zero), but two
//    calls whose kernels overlap on the GPU -- on different streams, or from
//    different host threads without ordering -- race on it. Order them.
//  * Nothing here allocates: no cudaMalloc, cudaFree or allocating library
//    routine is called.
#include <mutex>

#include "../../include/switchyard_b200.h"

#include <cuda_runtime.h>

namespace {

constexpr int64_t kNoAllocScratchFloats = int64_t(1) << 21;  // 8 MiB of fp32
constexpr int kMaxDevices = 64;

// The scratch itself. In host code this name is only a handle for the runtime
// (passing it to a kernel would pass a host address); the device address comes
// from cudaGetSymbolAddress below.
static __device__ __align__(256) float g_dw_scratch[kNoAllocScratchFloats];

// Device address of g_dw_scratch on the current device, looked up once per
// device and cached.
int scratch_address(float** out) {
  static std::mutex mu;
  static float* cache[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return SY_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return SY_ERR_CUDA;
  std::lock_guard<std::mutex> lk(mu);
  if (cache[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_dw_scratch);
    if (e != cudaSuccess || p == nullptr) return SY_ERR_CUDA;
    cache[dev] = static_cast<float*>(p);
  }
  *out = cache[dev];
  return SY_OK;
}

}  // namespace

extern "C" {

int64_t sy_bwd_noalloc_max_floats(void) { return kNoAllocScratchFloats; }

int sy_bwd_noalloc(const void* v, const void* w, const void* g, const float* stats, void* dv,
                   void* dw, int64_t N, int64_t BT, int64_t D, int dtype, int w_dtype, float eps,
                   sy_stream_t stream) {
  const int64_t P = sy_bwd_partials(N, BT, D, dtype);
  if (P < 1) return (int)-P;  // the same argument errors sy_bwd reports
  if (D > 0 && P > kNoAllocScratchFloats / D) return SY_ERR_SCRATCH;
  float* part = nullptr;
  const int st = scratch_address(&part);
  if (st != SY_OK) return st;
  const int sb = sy_bwd(v, w, g, stats, dv, part, P, N, BT, D, dtype, w_dtype, eps, stream);
  if (sb != SY_OK) return sb;
  return sy_dw_reduce(part, P, D, dw, w_dtype, stream);
}

}  // extern "C"
