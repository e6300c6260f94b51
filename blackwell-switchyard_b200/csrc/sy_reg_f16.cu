// sy_reg_f16.cu -- register-tile kernel instantiations for __half (N = 1..16).
// One file per dtype so nvcc compiles the three sets in parallel.
#include "sy_reg.cuh"

namespace sy {

cudaError_t launch_reg_fwd_f16(const TileCfg& c, int grid, int cpt, const void* v, const void* w,
                              int w_dtype, void* out, float* stats, cudaStream_t st) {
  return launch_reg_fwd_t<__half>(c, grid, cpt, v, w, w_dtype, out, stats, st);
}

cudaError_t launch_reg_bwd_f16(const TileCfg& c, int grid, int cpt, const void* v, const void* w,
                              int w_dtype, const void* g, const float* stats, void* dv, float* dwp,
                              cudaStream_t st) {
  return launch_reg_bwd_t<__half>(c, grid, cpt, v, w, w_dtype, g, stats, dv, dwp, st);
}

}  // namespace sy
