// sy_stream_batched.cu -- instantiations and launcher of the row-stream batched forward.
#include "sy_stream_batched.cuh"

namespace sy {

template <typename T>
static cudaError_t launch_stream_batched_t(const StreamBatchedCfg& c, int grid, const void* v,
                                           const void* q, void* out, cudaStream_t st) {
  if (c.warps * 32 > kStreamBatchedThreads) return cudaErrorInvalidConfiguration;
  const size_t smem = stream_batched_smem_layout(c).total;
  const T* vp = static_cast<const T*>(v);
  const T* qp = static_cast<const T*>(q);
  T* op = static_cast<T*>(out);
  if (c.S + 1 <= 16)
    return launch_smem(stream_batched_kernel<T, 16>, grid, dim3(c.warps * 32), smem, st, vp, qp,
                       op, c);
  return launch_smem(stream_batched_kernel<T, 32>, grid, dim3(c.warps * 32), smem, st, vp, qp, op,
                     c);
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
