// sy_launch.cuh -- host-side launch helper shared by the kernel files.
#pragma once

#include <cuda_runtime.h>

#include <mutex>
#include <set>
#include <utility>

namespace sy {

// Raise a kernel's dynamic shared-memory limit once per (kernel, device),
// then launch it on `st`. Returns the launch's error (cudaGetLastError), so a
// bad configuration is reported to the caller instead of being lost.
template <typename... KArgs, typename... Args>
cudaError_t launch_smem(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                        cudaStream_t st, Args&&... args) {
  // (kernel, device) -> largest dynamic smem size applied so far. Kernels with
  // identical signatures share this instantiation, hence the kernel key.
  static std::mutex mu;
  static std::set<std::pair<std::pair<const void*, int>, size_t>> raised;
  if (smem > 48 * 1024) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const void* key = reinterpret_cast<const void*>(kern);
    std::lock_guard<std::mutex> lk(mu);
    bool have = false;
    for (const auto& p : raised)
      if (p.first.first == key && p.first.second == dev && p.second >= smem) have = true;
    if (!have) {
      e = cudaFuncSetAttribute(key, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      raised.insert({{key, dev}, smem});
    }
  }
  kern<<<grid, block, smem, st>>>(static_cast<KArgs>(args)...);
  return cudaGetLastError();
}

}  // namespace sy
