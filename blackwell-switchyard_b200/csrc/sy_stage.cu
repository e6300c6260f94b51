// sy_stage.cu -- the decoder's arena staging step as one pass.
//
// After each sublayer the reference decoder updates the running block partial
// and copies it into the source arena (src/switchyard/model.py:532-535):
//
//   partial = partial + out              # elementwise add: 2 slabs read, 1 written
//   arena[len(blocks)].copy_(partial)    # copy: 1 slab read, 1 written
//
// Here both happen in one kernel: new_partial[i] = partial[i] + out[i] (fp32
// add, one rounding to the dtype -- what torch's add does for 16-bit types)
// is written to new_partial and to the arena slot. 2 slabs read, 2 written,
// one launch instead of two. 16-byte vector accesses when every pointer is
// 16-byte aligned and the length is a whole number of vectors, grid-striding
// over vectors; otherwise element by element.
#include "sy_launch.cuh"
#include "sy_tile.cuh"

namespace sy {

template <typename T>
__global__ void __launch_bounds__(256)
    stage_vec_kernel(const uint4* __restrict__ a, const uint4* __restrict__ b, uint4* __restrict__ c,
                     uint4* __restrict__ arena, long long nvec) {
  constexpr int P = Dt<T>::kVec / 2;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nvec;
       i += (long long)gridDim.x * blockDim.x) {
    float2 x[P], y[P];
    unpack2<T>(a[i], x);
    unpack2<T>(b[i], y);
#pragma unroll
    for (int k = 0; k < P; ++k) x[k] = make_float2(x[k].x + y[k].x, x[k].y + y[k].y);
    const uint4 r = pack2<T>(x);
    if (c != nullptr) c[i] = r;
    arena[i] = r;
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
    stage_scalar_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ c,
                        T* __restrict__ arena, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const T r = Dt<T>::from_f(Dt<T>::to_f(a[i]) + Dt<T>::to_f(b[i]));
    if (c != nullptr) c[i] = r;
    arena[i] = r;
  }
}

cudaError_t launch_stage(long long numel, int dtype, const void* partial, const void* out,
                         void* new_partial, void* arena, bool vec16, int grid, cudaStream_t st) {
  const int es = dtype == SY_F32 ? 4 : 2;
  if (vec16) {
    const long long nvec = numel * es / 16;
    const uint4* a = static_cast<const uint4*>(partial);
    const uint4* b = static_cast<const uint4*>(out);
    uint4* c = static_cast<uint4*>(new_partial);
    uint4* r = static_cast<uint4*>(arena);
    switch (dtype) {
      case SY_BF16:
        return launch_smem(stage_vec_kernel<__nv_bfloat16>, grid, 256, 0, st, a, b, c, r, nvec);
      case SY_F16:
        return launch_smem(stage_vec_kernel<__half>, grid, 256, 0, st, a, b, c, r, nvec);
      case SY_F32:
        return launch_smem(stage_vec_kernel<float>, grid, 256, 0, st, a, b, c, r, nvec);
      default:
        return cudaErrorInvalidValue;
    }
  }
  switch (dtype) {
    case SY_BF16: {
      using T = __nv_bfloat16;
      return launch_smem(stage_scalar_kernel<T>, grid, 256, 0, st, static_cast<const T*>(partial),
                         static_cast<const T*>(out), static_cast<T*>(new_partial),
                         static_cast<T*>(arena), numel);
    }
    case SY_F16: {
      using T = __half;
      return launch_smem(stage_scalar_kernel<T>, grid, 256, 0, st, static_cast<const T*>(partial),
                         static_cast<const T*>(out), static_cast<T*>(new_partial),
                         static_cast<T*>(arena), numel);
    }
    case SY_F32:
      return launch_smem(stage_scalar_kernel<float>, grid, 256, 0, st,
                         static_cast<const float*>(partial), static_cast<const float*>(out),
                         static_cast<float*>(new_partial), static_cast<float*>(arena), numel);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace sy
