// sy_batched_f32.cu -- batched-query register-tile kernel instantiations for float.
// One file per dtype so nvcc compiles the three sets in parallel.
#include "sy_batched.cuh"

namespace sy {

cudaError_t launch_batched_f32(const TileCfg& c, int grid, int cpt, int S, const void* v,
                             const void* q, void* out, cudaStream_t st) {
  return launch_batched_t<float>(c, grid, cpt, S, v, q, out, st);
}

}  // namespace sy
