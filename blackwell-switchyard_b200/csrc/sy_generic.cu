// sy_generic.cu -- kernels for shapes the tile kernels do not take: rows whose
// byte length is not a multiple of 16 (D = 63, 777, ...), pointers that are
// only element-aligned, or tiles too large for the shared-memory ring.
//
// One CTA (256 threads) per token, grid-striding over tokens. Pass 1 reads the
// rows with scalar coalesced loads and reduces per row (warp shuffle, then a
// fixed-order sum over the 8 warps in shared memory); pass 2 re-reads them,
// mostly from L2 (the rows of the CTAs in flight are far smaller than L2).
// Same math, fp32 accumulation, same statistics layout as the tile kernels.
#include "sy_launch.cuh"
#include "sy_tile.cuh"

namespace sy {

namespace {
constexpr int kGW = kGenericThreads / 32;  // warps per CTA
}

template <typename T>
__global__ void __launch_bounds__(kGenericThreads)
    gen_fwd_kernel(const T* __restrict__ v, const void* __restrict__ w, int w_dtype,
                   T* __restrict__ out, float* __restrict__ stats, int SW, long long BT, int N,
                   int D, float eps) {
  extern __shared__ float gsm[];
  float* part = gsm;               // [N][kGW][2]
  float* lgt = part + N * kGW * 2;  // [N]
  float* rr = lgt + N;             // [N]
  float* alpha = rr + N;           // [N]
  const int tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
  for (long long tok = blockIdx.x; tok < BT; tok += gridDim.x) {
    for (int n = 0; n < N; ++n) {
      const T* row = v + ((size_t)n * BT + tok) * D;
      float dot = 0.f, ssq = 0.f;
      for (int d = tid; d < D; d += kGenericThreads) {
        const float x = Dt<T>::to_f(row[d]);
        dot = fmaf(load_any(w, w_dtype, d), x, dot);
        ssq = fmaf(x, x, ssq);
      }
      dot = warp_sum(dot);
      ssq = warp_sum(ssq);
      if (lane == 0) {
        part[(n * kGW + wp) * 2] = dot;
        part[(n * kGW + wp) * 2 + 1] = ssq;
      }
    }
    __syncthreads();
    if (wp == 0) {
      float m = -INFINITY;
      for (int n = lane; n < N; n += 32) {
        float dot = 0.f, ssq = 0.f;
        for (int q = 0; q < kGW; ++q) {
          dot += part[(n * kGW + q) * 2];
          ssq += part[(n * kGW + q) * 2 + 1];
        }
        rr[n] = rsqrtf(ssq / (float)D + eps);
        lgt[n] = dot * rr[n];
        m = fmaxf(m, lgt[n]);
      }
      m = warp_max(m);
      float l = 0.f;
      for (int n = lane; n < N; n += 32) {
        alpha[n] = expf(lgt[n] - m);
        l += alpha[n];
      }
      l = warp_sum(l);
      const float inv = 1.f / l;
      for (int n = lane; n < N; n += 32) alpha[n] *= inv;
      if (stats != nullptr) {
        float* st = stats + tok * SW;
        for (int n = lane; n < N; n += 32) {
          st[n] = lgt[n];
          st[N + n] = rr[n];
        }
        if (lane == 0) {
          st[2 * N] = m;
          st[2 * N + 1] = m + logf(l);
        }
      }
    }
    __syncthreads();
    for (int d = tid; d < D; d += kGenericThreads) {
      float o = 0.f;
      for (int n = 0; n < N; ++n) o = fmaf(alpha[n], Dt<T>::to_f(v[((size_t)n * BT + tok) * D + d]), o);
      out[tok * D + d] = Dt<T>::from_f(o);
    }
    __syncthreads();
  }
}

template <typename T>
__global__ void __launch_bounds__(kGenericThreads)
    gen_sol_kernel(const T* __restrict__ v, T* __restrict__ out, long long BT, int N, int D) {
  for (long long tok = blockIdx.x; tok < BT; tok += gridDim.x)
    for (int d = threadIdx.x; d < D; d += kGenericThreads) {
      float o = 0.f;
      for (int n = 0; n < N; ++n) o += Dt<T>::to_f(v[((size_t)n * BT + tok) * D + d]);
      out[tok * D + d] = Dt<T>::from_f(o);
    }
}

// Backward: CTA b owns dw_partial row b and the tokens b, b+P, ... .
template <typename T>
__global__ void __launch_bounds__(kGenericThreads)
    gen_bwd_kernel(const T* __restrict__ v, const void* __restrict__ w, int w_dtype,
                   const T* __restrict__ g, const float* __restrict__ stats, int SW,
                   T* __restrict__ dv, float* __restrict__ dw_partial, long long BT, int N, int D,
                   float eps) {
  extern __shared__ float gsm[];
  float* part = gsm;               // [N][kGW]
  float* coef = part + N * kGW;    // [N][3]: alpha, da, 2*dssq
  const int tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
  float* prow = dw_partial + (size_t)blockIdx.x * D;
  for (int d = tid; d < D; d += kGenericThreads) prow[d] = 0.f;
  const float inv_d = 1.f / (float)D;
  for (long long tok = blockIdx.x; tok < BT; tok += gridDim.x) {
    const T* grow = g + tok * D;
    for (int n = 0; n < N; ++n) {
      const T* row = v + ((size_t)n * BT + tok) * D;
      float gs = 0.f;
      for (int d = tid; d < D; d += kGenericThreads)
        gs = fmaf(Dt<T>::to_f(grow[d]), Dt<T>::to_f(row[d]), gs);
      gs = warp_sum(gs);
      if (lane == 0) part[n * kGW + wp] = gs;
    }
    __syncthreads();
    if (wp == 0) {
      const float* st = stats + tok * SW;
      const float lse = st[2 * N + 1];
      float sacc = 0.f;
      for (int n = lane; n < N; n += 32) {
        float gsum = 0.f;
        for (int q = 0; q < kGW; ++q) gsum += part[n * kGW + q];
        const float al = expf(st[n] - lse);
        coef[n * 3] = al;
        coef[n * 3 + 1] = gsum;  // G_n, replaced below
        sacc += al * gsum;
      }
      const float S = warp_sum(sacc);
      for (int n = lane; n < N; n += 32) {
        const float al = coef[n * 3];
        const float dl = al * (coef[n * 3 + 1] - S);
        const float r = st[N + n];
        coef[n * 3 + 1] = dl * r;
        coef[n * 3 + 2] = -dl * st[n] * r * r * inv_d;
      }
    }
    __syncthreads();
    for (int d = tid; d < D; d += kGenericThreads) {
      const float gd = Dt<T>::to_f(grow[d]);
      const float wd = load_any(w, w_dtype, d);
      float acc = prow[d];
      for (int n = 0; n < N; ++n) {
        const size_t idx = ((size_t)n * BT + tok) * D + d;
        const float x = Dt<T>::to_f(v[idx]);
        const float al = coef[n * 3], da = coef[n * 3 + 1], cv = coef[n * 3 + 2];
        dv[idx] = Dt<T>::from_f(fmaf(cv, x, fmaf(da, wd, al * gd)));
        acc = fmaf(da, x, acc);
      }
      prow[d] = acc;
    }
    __syncthreads();
  }
}

// Batched forward for any shape: per token, all S*N query dots and the N sums
// of squares, then per query a softmax and a weighted sum.
template <typename T>
__global__ void __launch_bounds__(kGenericThreads)
    gen_batched_kernel(const T* __restrict__ v, const T* __restrict__ q, T* __restrict__ out,
                       long long BT, int N, int D, int S, float eps, float* __restrict__ mstats,
                       int raw) {
  extern __shared__ float gsm[];
  const int S1 = S + 1;
  float* part = gsm;                    // [N][S+1][kGW]   (index S = sum of squares)
  float* alpha = part + N * S1 * kGW;   // [S][N]
  const int tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
  for (long long tok = blockIdx.x; tok < BT; tok += gridDim.x) {
    for (int n = 0; n < N; ++n) {
      const T* row = v + ((size_t)n * BT + tok) * D;
      for (int s = 0; s <= S; ++s) {
        float acc = 0.f;
        for (int d = tid; d < D; d += kGenericThreads) {
          const float x = Dt<T>::to_f(row[d]);
          const float y = (s < S) ? Dt<T>::to_f(q[(size_t)s * D + d]) : x;
          acc = fmaf(y, x, acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) part[(n * S1 + s) * kGW + wp] = acc;
      }
    }
    __syncthreads();
    for (int s = wp; s < S; s += kGW) {
      float m = -INFINITY;
      for (int n = lane; n < N; n += 32) {
        float dot = 0.f, ssq = 0.f;
        for (int k = 0; k < kGW; ++k) {
          dot += part[(n * S1 + s) * kGW + k];
          ssq += part[(n * S1 + S) * kGW + k];
        }
        const float lg = dot * rsqrtf(ssq / (float)D + eps);
        alpha[s * N + n] = lg;
        m = fmaxf(m, lg);
      }
      m = warp_max(m);
      float l = 0.f;
      for (int n = lane; n < N; n += 32) {
        const float p = expf(alpha[s * N + n] - m);
        alpha[s * N + n] = p;
        l += p;
      }
      l = warp_sum(l);
      if (mstats != nullptr && lane == 0)
        reinterpret_cast<float2*>(mstats)[(size_t)s * BT + tok] = make_float2(m, l);
      if (!raw) {
        const float inv = 1.f / l;
        for (int n = lane; n < N; n += 32) alpha[s * N + n] *= inv;
      }
    }
    __syncthreads();
    for (int s = 0; s < S; ++s)
      for (int d = tid; d < D; d += kGenericThreads) {
        float o = 0.f;
        for (int n = 0; n < N; ++n)
          o = fmaf(alpha[s * N + n], Dt<T>::to_f(v[((size_t)n * BT + tok) * D + d]), o);
        out[((size_t)s * BT + tok) * D + d] = Dt<T>::from_f(o);
      }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
#define SY_DTYPE_SWITCH(dtype, T, ...)        \
  switch (dtype) {                            \
    case SY_BF16: {                           \
      using T = __nv_bfloat16;                \
      __VA_ARGS__;                            \
    }                                         \
    case SY_F16: {                            \
      using T = __half;                       \
      __VA_ARGS__;                            \
    }                                         \
    case SY_F32: {                            \
      using T = float;                        \
      __VA_ARGS__;                            \
    }                                         \
    default:                                  \
      return cudaErrorInvalidValue;           \
  }

cudaError_t launch_generic_fwd(long long BT, int N, int D, int dtype, const void* v,
                               const void* w, int w_dtype, void* out, float* stats,
                               int stats_stride, float eps, int grid, cudaStream_t st) {
  const size_t smem = ((size_t)N * kGW * 2 + 3 * (size_t)N) * sizeof(float);
  SY_DTYPE_SWITCH(dtype, T,
                  return launch_smem(gen_fwd_kernel<T>, grid, kGenericThreads, smem, st,
                                     static_cast<const T*>(v), w, w_dtype, static_cast<T*>(out),
                                     stats, stats_stride, BT, N, D, eps))
}

cudaError_t launch_generic_sol(long long BT, int N, int D, int dtype, const void* v, void* out,
                               int grid, cudaStream_t st) {
  SY_DTYPE_SWITCH(dtype, T,
                  return launch_smem(gen_sol_kernel<T>, grid, kGenericThreads, 0, st,
                                     static_cast<const T*>(v), static_cast<T*>(out), BT, N, D))
}

cudaError_t launch_generic_bwd(long long BT, int N, int D, int dtype, const void* v,
                               const void* w, int w_dtype, const void* g, const float* stats,
                               int stats_stride, void* dv, float* dw_partial, int P, float eps,
                               cudaStream_t st) {
  const size_t smem = ((size_t)N * kGW + 3 * (size_t)N) * sizeof(float);
  SY_DTYPE_SWITCH(dtype, T,
                  return launch_smem(gen_bwd_kernel<T>, P, kGenericThreads, smem, st,
                                     static_cast<const T*>(v), w, w_dtype,
                                     static_cast<const T*>(g), stats, stats_stride,
                                     static_cast<T*>(dv), dw_partial, BT, N, D, eps))
}

cudaError_t launch_generic_batched(long long BT, int N, int D, int S, int dtype, float* mstats,
                                   int raw, const void* v, const void* q, void* out, float eps,
                                   int grid, cudaStream_t st) {
  const size_t smem = ((size_t)N * (S + 1) * kGW + (size_t)S * N) * sizeof(float);
  SY_DTYPE_SWITCH(dtype, T,
                  return launch_smem(gen_batched_kernel<T>, grid, kGenericThreads, smem, st,
                                     static_cast<const T*>(v), static_cast<const T*>(q),
                                     static_cast<T*>(out), BT, N, D, S, eps, mstats, raw))
}

}  // namespace sy
