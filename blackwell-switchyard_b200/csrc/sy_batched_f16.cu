// sy_batched_f16.cu -- batched-query register-tile kernel instantiations for __half.
// One file per dtype so nvcc compiles the three sets in parallel.
#include "sy_batched.cuh"

namespace sy {

cudaError_t launch_batched_f16(const TileCfg& c, int grid, int cpt, int S, const void* v,
                             const void* q, void* out, cudaStream_t st) {
  return launch_batched_t<__half>(c, grid, cpt, S, v, q, out, st);
}

}  // namespace sy
