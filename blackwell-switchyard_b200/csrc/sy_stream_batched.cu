// sy_stream_batched.cu -- instantiations and launcher of the row-stream batched forward.
#include "sy_stream_batched.cuh"

namespace sy {

template <typename T, int SB, int CPL>
static cudaError_t launch_sb(const StreamBatchedCfg& c, int grid, const void* v, const void* q,
                             void* out, cudaStream_t st) {
  return launch_smem(stream_batched_kernel<T, SB, CPL>, grid, dim3(c.warps * 32),
                     stream_batched_smem_layout(c).total, st, static_cast<const T*>(v),
                     static_cast<const T*>(q), static_cast<T*>(out), c);
}

// (query slots, chunks per lane): the planner keeps SB * CPL <= 16 (the queries'
// registers in pass A).
template <typename T>
static cudaError_t launch_stream_batched_t(const StreamBatchedCfg& c, int grid, const void* v,
                                           const void* q, void* out, cudaStream_t st) {
  if (c.warps * 32 > kStreamBatchedThreads) return cudaErrorInvalidConfiguration;
  switch (c.sb * 8 + c.cpl) {
    case 4 * 8 + 2:
      return launch_sb<T, 4, 2>(c, grid, v, q, out, st);
    case 4 * 8 + 1:
      return launch_sb<T, 4, 1>(c, grid, v, q, out, st);
    case 8 * 8 + 2:
      return launch_sb<T, 8, 2>(c, grid, v, q, out, st);
    case 8 * 8 + 1:
      return launch_sb<T, 8, 1>(c, grid, v, q, out, st);
    case 16 * 8 + 1:
      return launch_sb<T, 16, 1>(c, grid, v, q, out, st);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_stream_batched(const StreamBatchedCfg& c, int grid, int dtype, const void* v,
                                  const void* q, void* out, cudaStream_t st) {
  switch (dtype) {
    case SY_BF16:
      return launch_stream_batched_t<__nv_bfloat16>(c, grid, v, q, out, st);
    case SY_F16:
      return launch_stream_batched_t<__half>(c, grid, v, q, out, st);
    case SY_F32:
      return launch_stream_batched_t<float>(c, grid, v, q, out, st);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace sy
