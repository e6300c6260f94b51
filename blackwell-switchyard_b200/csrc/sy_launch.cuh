// sy_launch.cuh -- host-side launch helpers shared by the kernel files.
#pragma once

#include <cuda_runtime.h>

#include <mutex>
#include <set>
#include <utility>

namespace sy {

// Raise a kernel's dynamic shared-memory limit once per (kernel, device).
template <typename... KArgs>
cudaError_t raise_smem_limit(void (*kern)(KArgs...), size_t smem) {
  if (smem <= 48 * 1024) return cudaSuccess;
  // (kernel, device) -> largest dynamic smem size applied so far. Kernels with
  // identical signatures share this instantiation, hence the kernel key.
  static std::mutex mu;
  static std::set<std::pair<std::pair<const void*, int>, size_t>> raised;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const void* key = reinterpret_cast<const void*>(kern);
  std::lock_guard<std::mutex> lk(mu);
  for (const auto& p : raised)
    if (p.first.first == key && p.first.second == dev && p.second >= smem) return cudaSuccess;
  e = cudaFuncSetAttribute(key, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  raised.insert({{key, dev}, smem});
  return cudaSuccess;
}

// Launch `kern` on `st` with `smem` bytes of dynamic shared memory. Returns the
// launch's error (cudaGetLastError), so a bad configuration is reported to the
// caller instead of being lost.
template <typename... KArgs, typename... Args>
cudaError_t launch_smem(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                        cudaStream_t st, Args&&... args) {
  cudaError_t e = raise_smem_limit(kern, smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, block, smem, st>>>(static_cast<KArgs>(args)...);
  return cudaGetLastError();
}

// As launch_smem, as a programmatic dependent launch: the kernel may start
// while the previous kernel on the stream finishes (its CTAs take the SMs that
// kernel's CTAs leave) and must execute `griddepcontrol.wait` before its first
// read of global memory, which returns once that kernel has completed and its
// writes are visible. The launch latency and the previous kernel's tail then
// overlap instead of adding up.
template <typename... KArgs, typename... Args>
cudaError_t launch_smem_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                            cudaStream_t st, Args&&... args) {
  cudaError_t e = raise_smem_limit(kern, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace sy
