// sy_batched_bf16.cu -- batched-query register-tile kernel instantiations for __nv_bfloat16.
// One file per dtype so nvcc compiles the three sets in parallel.
#include "sy_batched.cuh"

namespace sy {

cudaError_t launch_batched_bf16(const TileCfg& c, int grid, int cpt, int S, const void* v,
                             const void* q, void* out, cudaStream_t st) {
  return launch_batched_t<__nv_bfloat16>(c, grid, cpt, S, v, q, out, st);
}

}  // namespace sy
