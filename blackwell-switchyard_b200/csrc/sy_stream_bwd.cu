// sy_stream_bwd.cu -- instantiations and launcher of the row-stream backward.
#include "sy_stream_bwd.cuh"

namespace sy {

template <typename T, int SL, int CPL>
static cudaError_t launch_sb(const StreamBwdCfg& c, int grid, const void* v, const void* w,
                             int w_dtype, const void* g, const float* stats, void* dv,
                             float* dw_partial, cudaStream_t st) {
  return launch_smem_pdl(stream_bwd_kernel<T, SL, CPL>, grid, dim3(c.warps * 32),
                         stream_bwd_smem_layout(c).total, st, static_cast<const T*>(v), w, w_dtype,
                         static_cast<const T*>(g), stats, static_cast<T*>(dv), dw_partial, c);
}

template <typename T, int SL>
static cudaError_t launch_sb_cpl(const StreamBwdCfg& c, int grid, const void* v, const void* w,
                                 int w_dtype, const void* g, const float* stats, void* dv,
                                 float* dw_partial, cudaStream_t st) {
  switch (c.cpl) {
    case 1:
      return launch_sb<T, SL, 1>(c, grid, v, w, w_dtype, g, stats, dv, dw_partial, st);
    case 2:
      return launch_sb<T, SL, 2>(c, grid, v, w, w_dtype, g, stats, dv, dw_partial, st);
    case 4:
      return launch_sb<T, SL, 4>(c, grid, v, w, w_dtype, g, stats, dv, dw_partial, st);
    default:
      return cudaErrorInvalidValue;
  }
}

template <typename T>
static cudaError_t launch_stream_bwd_t(const StreamBwdCfg& c, int grid, const void* v,
                                       const void* w, int w_dtype, const void* g,
                                       const float* stats, void* dv, float* dw_partial,
                                       cudaStream_t st) {
  if (c.warps * 32 > kStreamBwdThreads) return cudaErrorInvalidConfiguration;
  if (c.N > 32)
    return launch_sb_cpl<T, 2>(c, grid, v, w, w_dtype, g, stats, dv, dw_partial, st);
  return launch_sb_cpl<T, 1>(c, grid, v, w, w_dtype, g, stats, dv, dw_partial, st);
}

cudaError_t launch_stream_bwd(const StreamBwdCfg& c, int grid, int dtype, const void* v,
                              const void* w, int w_dtype, const void* g, const float* stats,
                              void* dv, float* dw_partial, cudaStream_t st) {
  switch (dtype) {
    case SY_BF16:
      return launch_stream_bwd_t<__nv_bfloat16>(c, grid, v, w, w_dtype, g, stats, dv, dw_partial,
                                                st);
    case SY_F16:
      return launch_stream_bwd_t<__half>(c, grid, v, w, w_dtype, g, stats, dv, dw_partial, st);
    case SY_F32:
      return launch_stream_bwd_t<float>(c, grid, v, w, w_dtype, g, stats, dv, dw_partial, st);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace sy
