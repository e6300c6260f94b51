// sy_batched_bwd.cu -- backward of the batched-query operator and the
// online-softmax merge of two partial results.
//
// Batched forward (block_attn_res_batched, src/switchyard/triton_op.py:438-501,
// forward only in the reference): for queries q_s and sources v_n of a token,
//
//   r_n = rsqrt(mean(v_n^2) + eps),  a_{s,n} = q_s . v_n,  logit = a r_n,
//   alpha_{s,n} = exp(logit_{s,n} - m_s) / l_s,  out_s = sum_n alpha_{s,n} v_n.
//
// With g_s the gradient of out_s, G_{s,n} = g_s . v_n, delta_s = sum_n alpha G:
//
//   dlogit_{s,n} = alpha_{s,n} (G_{s,n} - delta_s),   da_{s,n} = dlogit r_n,
//   dv_n = sum_s alpha_{s,n} g_s + sum_s da_{s,n} q_s + cv_n v_n,
//          cv_n = -sum_s dlogit_{s,n} logit_{s,n} r_n^2 / D,
//   dq_s = sum over tokens of sum_n da_{s,n} v_n.
//
// The backward recomputes the dot products from v (one pass over the token's
// rows, every a, G and sum of squares together) and the softmax from them, so
// it needs nothing from the forward but v and q, and the only large tensors
// are v, g and dv. One CTA owns a
// token at a time and one fp32 dq partial row [S, D] (its tokens b, b + P, ...);
// sy_dw_reduce sums the P rows in a fixed order, so dq is deterministic.
//
// The merge is Algorithm 1 line 12 of the paper (merge_online_softmax,
// src/switchyard/reference.py:219-233) on (o, m, l) triples, one CTA per row,
// with the final o / l division optionally fused.
#include "sy_launch.cuh"
#include "sy_tile.cuh"

namespace sy {

namespace {
constexpr int kBW = kGenericThreads / 32;  // warps per CTA
constexpr int kBwdBatchedMaxS = 16;
}  // namespace

// Shared memory: part [N][2S+1][kBW] (per-warp dot partials), alpha [S][N],
// da [S][N], cvp [S][N] (per-query terms of cv_n), cv [N], r [N].
template <typename T>
__global__ void __launch_bounds__(kGenericThreads)
    bat_bwd_kernel(const T* __restrict__ v, const T* __restrict__ q, const T* __restrict__ g,
                   T* __restrict__ dv,
                   float* __restrict__ dq_partial, long long BT, int N, int D, int S, float eps) {
  extern __shared__ float bsm[];
  const int L = 2 * S + 1;
  float* part = bsm;                          // [N][L][kBW]
  float* alpha = part + (size_t)N * L * kBW;  // [S][N]
  float* dam = alpha + S * N;                 // [S][N]
  float* cvp = dam + S * N;                   // [S][N]
  float* cv = cvp + S * N;                    // [N]
  float* rr = cv + N;                         // [N]
  const int tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
  float* prow = dq_partial + (size_t)blockIdx.x * S * D;
  for (int i = tid; i < S * D; i += kGenericThreads) prow[i] = 0.f;
  const float inv_d = 1.f / (float)D;
  for (long long tok = blockIdx.x; tok < BT; tok += gridDim.x) {
    // ---- every dot product of the token: a_{s,n}, G_{s,n}, ssq_n ----
    for (int n = 0; n < N; ++n) {
      const T* row = v + ((size_t)n * BT + tok) * D;
      float aq[kBwdBatchedMaxS], ag[kBwdBatchedMaxS], sq = 0.f;
#pragma unroll
      for (int j = 0; j < kBwdBatchedMaxS; ++j) aq[j] = ag[j] = 0.f;
      for (int d = tid; d < D; d += kGenericThreads) {
        const float x = Dt<T>::to_f(row[d]);
#pragma unroll
        for (int j = 0; j < kBwdBatchedMaxS; ++j) {
          if (j < S) {
            aq[j] = fmaf(Dt<T>::to_f(q[(size_t)j * D + d]), x, aq[j]);
            ag[j] = fmaf(Dt<T>::to_f(g[((size_t)j * BT + tok) * D + d]), x, ag[j]);
          }
        }
        sq = fmaf(x, x, sq);
      }
      float* pn = part + (size_t)n * L * kBW + wp;
#pragma unroll
      for (int j = 0; j < kBwdBatchedMaxS; ++j) {
        if (j < S) {  // warp-uniform
          const float ta = warp_sum(aq[j]);
          const float tg = warp_sum(ag[j]);
          if (lane == 0) {
            pn[(size_t)j * kBW] = ta;
            pn[(size_t)(S + j) * kBW] = tg;
          }
        }
      }
      const float ts = warp_sum(sq);
      if (lane == 0) pn[(size_t)(L - 1) * kBW] = ts;
    }
    __syncthreads();
    for (int n = tid; n < N; n += kGenericThreads) {
      float ssq = 0.f;
      for (int k = 0; k < kBW; ++k) ssq += part[((size_t)n * L + L - 1) * kBW + k];
      rr[n] = rsqrtf(ssq * inv_d + eps);
    }
    __syncthreads();
    // ---- per query: the softmax recomputed from the logits (so the weights
    //      are those of this pass's logits, and sum to 1), then the
    //      coefficients; warp w takes queries w, w + 8, ...; lane n source n ----
    for (int s = wp; s < S; s += kBW) {
      float mloc = -INFINITY;
      for (int n = lane; n < N; n += 32) {
        float a = 0.f;
        for (int k = 0; k < kBW; ++k) a += part[((size_t)n * L + s) * kBW + k];
        const float lg = a * rr[n];
        cvp[s * N + n] = lg;  // replaced below
        mloc = fmaxf(mloc, lg);
      }
      const float m = warp_max(mloc);
      float lsum = 0.f;
      for (int n = lane; n < N; n += 32) {
        const float e = expf(cvp[s * N + n] - m);
        alpha[s * N + n] = e;
        lsum += e;
      }
      const float inv_l = 1.f / warp_sum(lsum);
      float dsum = 0.f;
      for (int n = lane; n < N; n += 32) {
        float G = 0.f;
        for (int k = 0; k < kBW; ++k) G += part[((size_t)n * L + S + s) * kBW + k];
        const float al = alpha[s * N + n] * inv_l;
        alpha[s * N + n] = al;
        dam[s * N + n] = G;  // replaced below
        dsum += al * G;
      }
      const float delta = warp_sum(dsum);
      for (int n = lane; n < N; n += 32) {
        const float r = rr[n];
        const float dl = alpha[s * N + n] * (dam[s * N + n] - delta);
        dam[s * N + n] = dl * r;
        cvp[s * N + n] = -dl * cvp[s * N + n] * r * r * inv_d;
      }
    }
    __syncthreads();
    for (int n = tid; n < N; n += kGenericThreads) {
      float c = 0.f;
      for (int s = 0; s < S; ++s) c += cvp[s * N + n];
      cv[n] = c;
    }
    __syncthreads();
    // ---- dv and the dq partial row ----
    for (int d = tid; d < D; d += kGenericThreads) {
      float gd[kBwdBatchedMaxS], qd[kBwdBatchedMaxS], dq[kBwdBatchedMaxS];
#pragma unroll
      for (int s = 0; s < kBwdBatchedMaxS; ++s) {
        gd[s] = s < S ? Dt<T>::to_f(g[((size_t)s * BT + tok) * D + d]) : 0.f;
        qd[s] = s < S ? Dt<T>::to_f(q[(size_t)s * D + d]) : 0.f;
        dq[s] = s < S ? prow[(size_t)s * D + d] : 0.f;
      }
      for (int n = 0; n < N; ++n) {
        const size_t idx = ((size_t)n * BT + tok) * D + d;
        const float x = Dt<T>::to_f(v[idx]);
        float acc = cv[n] * x;
#pragma unroll
        for (int s = 0; s < kBwdBatchedMaxS; ++s) {
          if (s < S) {
            const float da = dam[s * N + n];
            acc = fmaf(alpha[s * N + n], gd[s], acc);
            acc = fmaf(da, qd[s], acc);
            dq[s] = fmaf(da, x, dq[s]);
          }
        }
        dv[idx] = Dt<T>::from_f(acc);
      }
#pragma unroll
      for (int s = 0; s < kBwdBatchedMaxS; ++s)
        if (s < S) prow[(size_t)s * D + d] = dq[s];
    }
    __syncthreads();
  }
}

size_t bwd_batched_smem(int N, int S) {
  return ((size_t)N * (2 * S + 1) * kBW + 3 * (size_t)S * N + 2 * (size_t)N) * sizeof(float);
}

// Merge two partial results over disjoint source groups (per row: o [D],
// (m, l)). m = max(m1, m2), s_i = exp(m_i - m), o = o1 s1 + o2 s2,
// l = l1 s1 + l2 s2; normalize = 1 writes o / l instead of o.
template <typename T>
__global__ void __launch_bounds__(kGenericThreads)
    merge_kernel(const T* __restrict__ o1, const float* __restrict__ ms1, const T* __restrict__ o2,
                 const float* __restrict__ ms2, T* __restrict__ o, float* __restrict__ ms,
                 long long R, int D, int normalize) {
  for (long long row = blockIdx.x; row < R; row += gridDim.x) {
    const float2 a = reinterpret_cast<const float2*>(ms1)[row];
    const float2 b = reinterpret_cast<const float2*>(ms2)[row];
    const float m = fmaxf(a.x, b.x);
    const float s1 = expf(a.x - m), s2 = expf(b.x - m);
    const float l = a.y * s1 + b.y * s2;
    float c1 = s1, c2 = s2;
    if (normalize) {
      const float inv = 1.f / l;
      c1 *= inv;
      c2 *= inv;
    }
    const size_t base = (size_t)row * D;
    for (int d = threadIdx.x; d < D; d += kGenericThreads)
      o[base + d] = Dt<T>::from_f(
          fmaf(Dt<T>::to_f(o1[base + d]), c1, Dt<T>::to_f(o2[base + d]) * c2));
    if (ms != nullptr && threadIdx.x == 0)
      reinterpret_cast<float2*>(ms)[row] = make_float2(m, l);
  }
}

#define SY_BB_DTYPE_SWITCH(dtype, T, ...) \
  switch (dtype) {                        \
    case SY_BF16: {                       \
      using T = __nv_bfloat16;            \
      __VA_ARGS__;                        \
    }                                     \
    case SY_F16: {                        \
      using T = __half;                   \
      __VA_ARGS__;                        \
    }                                     \
    case SY_F32: {                        \
      using T = float;                    \
      __VA_ARGS__;                        \
    }                                     \
    default:                              \
      return cudaErrorInvalidValue;       \
  }

cudaError_t launch_bwd_batched(long long BT, int N, int D, int S, int dtype, const void* v,
                               const void* q, const void* g, void* dv, float* dq_partial, int P,
                               float eps, cudaStream_t st) {
  if (S < 1 || S > kBwdBatchedMaxS) return cudaErrorInvalidValue;
  const size_t smem = bwd_batched_smem(N, S);
  SY_BB_DTYPE_SWITCH(dtype, T,
                     return launch_smem(bat_bwd_kernel<T>, P, kGenericThreads, smem, st,
                                        static_cast<const T*>(v), static_cast<const T*>(q),
                                        static_cast<const T*>(g), static_cast<T*>(dv),
                                        dq_partial, BT, N, D, S, eps))
}

cudaError_t launch_merge(long long R, int D, int dtype, const void* o1, const float* ms1,
                         const void* o2, const float* ms2, void* o, float* ms, int normalize,
                         int grid, cudaStream_t st) {
  SY_BB_DTYPE_SWITCH(dtype, T,
                     return launch_smem(merge_kernel<T>, grid, kGenericThreads, 0, st,
                                        static_cast<const T*>(o1), ms1,
                                        static_cast<const T*>(o2), ms2, static_cast<T*>(o), ms, R,
                                        D, normalize))
}

}  // namespace sy
