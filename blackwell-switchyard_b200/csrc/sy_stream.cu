// sy_stream.cu -- instantiations and launcher of the row-stream forward.
#include "sy_stream.cuh"

namespace sy {

cudaError_t launch_stream_fwd(const StreamCfg& c, int grid, int cpl, int dtype, const void* v,
                              const void* w, int w_dtype, void* out, float* stats, bool sol,
                              cudaStream_t st) {
  switch (dtype) {
    case SY_BF16:
      return sol ? launch_stream_t<__nv_bfloat16, true>(c, grid, cpl, v, w, w_dtype, out, stats, st)
                 : launch_stream_t<__nv_bfloat16, false>(c, grid, cpl, v, w, w_dtype, out, stats, st);
    case SY_F16:
      return sol ? launch_stream_t<__half, true>(c, grid, cpl, v, w, w_dtype, out, stats, st)
                 : launch_stream_t<__half, false>(c, grid, cpl, v, w, w_dtype, out, stats, st);
    case SY_F32:
      return sol ? launch_stream_t<float, true>(c, grid, cpl, v, w, w_dtype, out, stats, st)
                 : launch_stream_t<float, false>(c, grid, cpl, v, w, w_dtype, out, stats, st);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace sy
