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
#include "sy_reg.cuh"
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

// ---------------------------------------------------------------------------
// Register-tile variant for rows of at most 256 16-byte chunks (4 KiB) and
// N <= kBwdRegMaxN: thread t owns chunk t of every row of the token, so the
// token's N source chunks are read from HBM once, into registers, and every
// dot product, dv and the thread's columns of dq come from them.
//
//   * sums of squares: one 16-value reduce-scatter per warp;
//   * per query s: q_s . v_n and g_s . v_n (packed 16-bit FMA into fp32) for
//     all n, one 32-value reduce-scatter (values 0..15: q dots, 16..31: g dots);
//     warp totals to shared memory, summed over the 8 warps in warp order;
//   * coefficients: warp w takes queries w, w + 8, ...; lane n source n;
//   * dv_n = sum_s (alpha_{s,n} g_s + da_{s,n} q_s) + cv_n v_n in fp32
//     registers, one rounding; dq_s's columns of this thread accumulate in
//     shared memory (thread-private, no barrier) over the CTA's tokens and are
//     written once as the CTA's partial row.
// ---------------------------------------------------------------------------
constexpr int kBwdRegMaxN = 9;
constexpr int kRegBwdStaged = 3;  // reg_bwd_batched_variant: the staged kernel
#ifndef SY_TUNE_BWD_STAGED_MIN_S
#define SY_TUNE_BWD_STAGED_MIN_S 1  // smallest S the staged kernel takes
#endif
int reg_bwd_batched_ctas_per_sm(int N, int D, int S, int dtype, int max_smem);  // no spills for any dtype up to here (fp16 spills from 10)

template <typename T>
__device__ __forceinline__ float dot_chunk(const uint4& a, const uint4& b) {
  if constexpr (sizeof(T) == 2) {
    float2 acc = make_float2(0.f, 0.f);
    mixfma2<T>(acc, a.x, b.x);
    mixfma2<T>(acc, a.y, b.y);
    mixfma2<T>(acc, a.z, b.z);
    mixfma2<T>(acc, a.w, b.w);
    return acc.x + acc.y;
  } else {
    const float4 x = *reinterpret_cast<const float4*>(&a);
    const float4 y = *reinterpret_cast<const float4*>(&b);
    float2 acc = make_float2(x.x * y.x, x.y * y.y);
    acc = __ffma2_rn(make_float2(x.z, x.w), make_float2(y.z, y.w), acc);
    return acc.x + acc.y;
  }
}

struct RegBwdSmem {
  size_t q_off, dq_off, red_off, coef_off, cvp_off, total;
};
__host__ __device__ inline RegBwdSmem reg_bwd_batched_layout(int N, int S, int rc, int vec) {
  RegBwdSmem L;
  L.q_off = 0;                                                   // [S][rc] uint4
  L.dq_off = L.q_off + (size_t)S * rc * 16;                      // [S][rc * vec] fp32
  L.red_off = L.dq_off + (size_t)S * rc * vec * 4;               // [S + 1][8][32] fp32
  L.coef_off = L.red_off + (size_t)(S + 1) * kBW * 32 * 4;      // [S][N] float2
  L.cvp_off = L.coef_off + (size_t)S * N * 8;                    // [S][N] fp32
  L.total = L.cvp_off + (size_t)S * N * 4;
  return L;
}

template <typename T, int N, int MINB>
__global__ void __launch_bounds__(kGenericThreads, MINB)
    reg_bat_bwd_kernel(const T* __restrict__ v, const T* __restrict__ q, const T* __restrict__ g,
                       T* __restrict__ dv, float* __restrict__ dq_partial, long long BT, int D,
                       int S, int rc, float eps) {
  constexpr int VEC = Dt<T>::kVec;
  constexpr int P = VEC / 2;
  extern __shared__ __align__(16) unsigned char rsm[];
  const RegBwdSmem L = reg_bwd_batched_layout(N, S, rc, VEC);
  uint4* qs = reinterpret_cast<uint4*>(rsm + L.q_off);
  float* dqs = reinterpret_cast<float*>(rsm + L.dq_off);
  float* red = reinterpret_cast<float*>(rsm + L.red_off);
  float2* coef = reinterpret_cast<float2*>(rsm + L.coef_off);
  float* cvp = reinterpret_cast<float*>(rsm + L.cvp_off);
  const int tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
  const bool act = tid < rc;
  const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
  for (int i = tid; i < S * rc; i += kGenericThreads)
    qs[i] = reinterpret_cast<const uint4*>(q)[i];
  for (int i = tid; i < S * rc * VEC; i += kGenericThreads) dqs[i] = 0.f;
  __syncthreads();
  const float inv_d = 1.f / (float)D;
  for (long long tok = blockIdx.x; tok < BT; tok += gridDim.x) {
    uint4 vx[N];
#pragma unroll
    for (int n = 0; n < N; ++n)
      vx[n] = act ? reinterpret_cast<const uint4*>(v + ((size_t)n * BT + tok) * D)[tid] : z4;
    {
      float sv[16];
#pragma unroll
      for (int n = 0; n < 16; ++n) sv[n] = n < N ? dot_chunk<T>(vx[n], vx[n]) : 0.f;
      const float t = warp_reduce_scatter16(sv, lane);
      if ((lane & 1) == 0 && (lane >> 1) < N) red[((size_t)S * kBW + wp) * 32 + (lane >> 1)] = t;
    }
    // g_{s+1}'s chunk is requested before g_s's dots are reduced (one query
    // ahead), so its latency overlaps the reduction instead of following it
    const uint4* gcol = reinterpret_cast<const uint4*>(g + (size_t)tok * D) + tid;
    const size_t gstride = (size_t)BT * D / Dt<T>::kVec;  // one query's slab, in chunks
    uint4 gnext = act ? gcol[0] : z4;
    for (int s = 0; s < S; ++s) {
      const uint4 gx = gnext;
      if (act && s + 1 < S) gnext = gcol[(size_t)(s + 1) * gstride];
      const uint4 qx = act ? qs[s * rc + tid] : z4;
      float a[32];
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        a[n] = n < N ? dot_chunk<T>(qx, vx[n]) : 0.f;
        a[16 + n] = n < N ? dot_chunk<T>(gx, vx[n]) : 0.f;
      }
      const float t = warp_reduce_scatter<32>(a, lane);
      if ((lane & 15) < N) red[((size_t)s * kBW + wp) * 32 + lane] = t;
    }
    __syncthreads();
    for (int s = wp; s < S; s += kBW) {
      const bool on = lane < N;
      const int n = on ? lane : 0;
      float a = 0.f, G = 0.f, ssq = 0.f;
      for (int k = 0; k < kBW; ++k) {
        a += red[((size_t)s * kBW + k) * 32 + n];
        G += red[((size_t)s * kBW + k) * 32 + 16 + n];
        ssq += red[((size_t)S * kBW + k) * 32 + n];
      }
      const float r = rsqrtf(ssq * inv_d + eps);
      const float lg = a * r;
      const float m = warp_max(on ? lg : -INFINITY);
      const float e = on ? expf(lg - m) : 0.f;
      const float al = e / warp_sum(e);
      const float delta = warp_sum(on ? al * G : 0.f);
      const float dl = al * (G - delta);
      if (on) {
        coef[s * N + n] = make_float2(al, dl * r);
        cvp[s * N + n] = -dl * lg * r * r * inv_d;
      }
    }
    __syncthreads();
    // MINB = 2: dv in two halves of the chunk (H float2 pairs each), so only
    // N * H fp32 pairs of accumulators are live and two CTAs fit an SM's
    // registers; g_s is re-read per half (from L2), q_s from shared memory.
    // MINB = 1 (shared memory holds one CTA anyway): the whole chunk at once.
    constexpr int H = (MINB == 2 && P / 2 > 0) ? P / 2 : P;
    float cvn[N];
#pragma unroll
    for (int n = 0; n < N; ++n) cvn[n] = 0.f;
#pragma unroll
    for (int h = 0; h < P / H; ++h) {
      float2 acc[N][H];
#pragma unroll
      for (int n = 0; n < N; ++n)
#pragma unroll
        for (int i = 0; i < H; ++i) acc[n][i] = make_float2(0.f, 0.f);
      gnext = act ? gcol[0] : z4;
      for (int s = 0; s < S; ++s) {
        const uint4 gx = gnext;
        if (act && s + 1 < S) gnext = gcol[(size_t)(s + 1) * gstride];
        const uint4 qx = act ? qs[s * rc + tid] : z4;
        float2 gf[P], qf[P], dqp[H];
        unpack2<T>(gx, gf);
        unpack2<T>(qx, qf);
#pragma unroll
        for (int i = 0; i < H; ++i) dqp[i] = make_float2(0.f, 0.f);
#pragma unroll
        for (int n = 0; n < N; ++n) {
          const float2 cf = coef[s * N + n];
          if (h == 0) cvn[n] += cvp[s * N + n];
          float2 vf[P];
          unpack2<T>(vx[n], vf);
#pragma unroll
          for (int i = 0; i < H; ++i) {
            acc[n][i] = __ffma2_rn(f2(cf.x), gf[h * H + i], acc[n][i]);
            acc[n][i] = __ffma2_rn(f2(cf.y), qf[h * H + i], acc[n][i]);
            dqp[i] = __ffma2_rn(f2(cf.y), vf[h * H + i], dqp[i]);
          }
        }
        if (act) {
          float2* dq2 =
              reinterpret_cast<float2*>(dqs + (size_t)s * rc * VEC + (size_t)tid * VEC) + h * H;
#pragma unroll
          for (int i = 0; i < H; ++i) {
            const float2 o = dq2[i];
            dq2[i] = make_float2(o.x + dqp[i].x, o.y + dqp[i].y);
          }
        }
      }
      if (act) {
#pragma unroll
        for (int n = 0; n < N; ++n) {
          float2 vf[P];
          unpack2<T>(vx[n], vf);
          float2 o[P];
#pragma unroll
          for (int i = 0; i < P; ++i) o[i] = make_float2(0.f, 0.f);
#pragma unroll
          for (int i = 0; i < H; ++i) o[h * H + i] = __ffma2_rn(f2(cvn[n]), vf[h * H + i], acc[n][i]);
          const uint4 pk = pack2<T>(o);
          if constexpr (H == P) {  // the whole 16-byte chunk
            reinterpret_cast<uint4*>(dv + ((size_t)n * BT + tok) * D)[tid] = pk;
          } else {  // this half's 8 bytes of the 16-byte chunk
            uint2* dst = reinterpret_cast<uint2*>(dv + ((size_t)n * BT + tok) * D) + 2 * tid + h;
            *dst = h == 0 ? make_uint2(pk.x, pk.y) : make_uint2(pk.z, pk.w);
          }
        }
      }
    }
  }
  if (act) {
    float* prow = dq_partial + (size_t)blockIdx.x * S * D;
    for (int s = 0; s < S; ++s) {
      const float4* src = reinterpret_cast<const float4*>(dqs + (size_t)s * rc * VEC + (size_t)tid * VEC);
      float4* dst = reinterpret_cast<float4*>(prow + (size_t)s * D + (size_t)tid * VEC);
#pragma unroll
      for (int i = 0; i < VEC / 4; ++i) dst[i] = src[i];
    }
  }
}

// ---------------------------------------------------------------------------
// Staged variant (S <= 8 at 4 KiB rows; one CTA of 8 warps per SM): the
// token's N source chunks unpacked to fp32 once (N x VEC floats a thread, so
// every dot product and dv term comes from registers and dv is one pass over
// the queries), the next token's source chunks requested into registers and
// its g chunks copied into shared memory (cp.async, two buffers) at the start
// of this token, so neither waits on HBM. A thread copies and reads only its
// own chunk positions, so the copies need no barrier: it waits for its own
// previous copy group. The numbers are the same as the half-pass kernel's
// (same per-element operation order), except for the dq partial-row count.
// ---------------------------------------------------------------------------
__host__ __device__ inline size_t reg_bwd_staged_g_off(int N, int S, int rc, int vec) {
  return (reg_bwd_batched_layout(N, S, rc, vec).total + 15) / 16 * 16;
}
__host__ __device__ inline size_t reg_bwd_staged_total(int N, int S, int rc, int vec) {
  return reg_bwd_staged_g_off(N, S, rc, vec) + (size_t)2 * S * rc * 16;  // [2][S][rc] uint4
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// All but the most recent of this thread's copy groups have landed.
__device__ __forceinline__ void cp_async_wait_prev() {
  asm volatile("cp.async.wait_group 1;" ::: "memory");
}

// The packed dot product of two unpacked chunks: even and odd elements in the
// two lanes of one fp32 pair, added once (the same order as dot_chunk).
template <int P>
__device__ __forceinline__ float dot_pairs(const float2 (&a)[P], const float2 (&b)[P]) {
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < P; ++i) acc = __ffma2_rn(a[i], b[i], acc);
  return acc.x + acc.y;
}

template <typename T, int N>
__global__ void __launch_bounds__(kGenericThreads, 1)
    reg_bat_bwd_staged_kernel(const T* __restrict__ v, const T* __restrict__ q,
                              const T* __restrict__ g, T* __restrict__ dv,
                              float* __restrict__ dq_partial, long long BT, int D, int S, int rc,
                              float eps) {
  constexpr int VEC = Dt<T>::kVec;
  constexpr int P = VEC / 2;
  extern __shared__ __align__(16) unsigned char rsm[];
  const RegBwdSmem L = reg_bwd_batched_layout(N, S, rc, VEC);
  uint4* qs = reinterpret_cast<uint4*>(rsm + L.q_off);
  float* dqs = reinterpret_cast<float*>(rsm + L.dq_off);
  float* red = reinterpret_cast<float*>(rsm + L.red_off);
  float2* coef = reinterpret_cast<float2*>(rsm + L.coef_off);
  float* cvp = reinterpret_cast<float*>(rsm + L.cvp_off);
  uint4* gbuf = reinterpret_cast<uint4*>(rsm + reg_bwd_staged_g_off(N, S, rc, VEC));
  const int tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
  const bool act = tid < rc;
  const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
  for (int i = tid; i < S * rc; i += kGenericThreads)
    qs[i] = reinterpret_cast<const uint4*>(q)[i];
  for (int i = tid; i < S * rc * VEC; i += kGenericThreads) dqs[i] = 0.f;
  __syncthreads();
  const float inv_d = 1.f / (float)D;
  const size_t gstride = (size_t)BT * D / VEC;  // one query's slab of g, in chunks
  // this thread's chunk of every query's g row of token `tk`, into buffer `bi`;
  // every thread commits a group (an empty one when it copies nothing)
  auto stage_g = [&](long long tk, int bi) {
    if (act && tk < BT) {
      const uint4* src = reinterpret_cast<const uint4*>(g + (size_t)tk * D) + tid;
      uint4* dst = gbuf + (size_t)bi * S * rc + tid;
      for (int s = 0; s < S; ++s) cp_async16(dst + (size_t)s * rc, src + (size_t)s * gstride);
    }
    cp_async_commit();
  };
  uint4 vn[N];  // the raw source chunks of the next token
#pragma unroll
  for (int n = 0; n < N; ++n)
    vn[n] = act && (long long)blockIdx.x < BT
                ? reinterpret_cast<const uint4*>(v + ((size_t)n * BT + blockIdx.x) * D)[tid]
                : z4;
  stage_g(blockIdx.x, 0);
  int j = 0;
  for (long long tok = blockIdx.x; tok < BT; tok += gridDim.x, ++j) {
    float2 vf[N][P];
#pragma unroll
    for (int n = 0; n < N; ++n) unpack2<T>(vn[n], vf[n]);
    const long long nxt = tok + gridDim.x;
#pragma unroll
    for (int n = 0; n < N; ++n)
      vn[n] = act && nxt < BT
                  ? reinterpret_cast<const uint4*>(v + ((size_t)n * BT + nxt) * D)[tid]
                  : z4;
    stage_g(nxt, (j + 1) & 1);
    cp_async_wait_prev();  // this token's g chunks have landed
    const uint4* gtok = gbuf + (size_t)(j & 1) * S * rc + tid;
    {
      float sv[16];
#pragma unroll
      for (int n = 0; n < 16; ++n) sv[n] = n < N ? dot_pairs<P>(vf[n], vf[n]) : 0.f;
      const float t = warp_reduce_scatter16(sv, lane);
      if ((lane & 1) == 0 && (lane >> 1) < N) red[((size_t)S * kBW + wp) * 32 + (lane >> 1)] = t;
    }
    for (int s = 0; s < S; ++s) {
      const uint4 gx = act ? gtok[(size_t)s * rc] : z4;
      const uint4 qx = act ? qs[s * rc + tid] : z4;
      float2 gf[P], qf[P];
      unpack2<T>(gx, gf);
      unpack2<T>(qx, qf);
      float a[32];
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        a[n] = n < N ? dot_pairs<P>(qf, vf[n]) : 0.f;
        a[16 + n] = n < N ? dot_pairs<P>(gf, vf[n]) : 0.f;
      }
      const float t = warp_reduce_scatter<32>(a, lane);
      if ((lane & 15) < N) red[((size_t)s * kBW + wp) * 32 + lane] = t;
    }
    __syncthreads();
    for (int s = wp; s < S; s += kBW) {
      const bool on = lane < N;
      const int n = on ? lane : 0;
      float a = 0.f, G = 0.f, ssq = 0.f;
      for (int k = 0; k < kBW; ++k) {
        a += red[((size_t)s * kBW + k) * 32 + n];
        G += red[((size_t)s * kBW + k) * 32 + 16 + n];
        ssq += red[((size_t)S * kBW + k) * 32 + n];
      }
      const float r = rsqrtf(ssq * inv_d + eps);
      const float lg = a * r;
      const float m = warp_max(on ? lg : -INFINITY);
      const float e = on ? expf(lg - m) : 0.f;
      const float al = e / warp_sum(e);
      const float delta = warp_sum(on ? al * G : 0.f);
      const float dl = al * (G - delta);
      if (on) {
        coef[s * N + n] = make_float2(al, dl * r);
        cvp[s * N + n] = -dl * lg * r * r * inv_d;
      }
    }
    __syncthreads();
    float2 acc[N][P];
    float cvn[N];
#pragma unroll
    for (int n = 0; n < N; ++n) {
      cvn[n] = 0.f;
#pragma unroll
      for (int i = 0; i < P; ++i) acc[n][i] = make_float2(0.f, 0.f);
    }
    for (int s = 0; s < S; ++s) {
      const uint4 gx = act ? gtok[(size_t)s * rc] : z4;
      const uint4 qx = act ? qs[s * rc + tid] : z4;
      float2 gf[P], qf[P], dqp[P];
      unpack2<T>(gx, gf);
      unpack2<T>(qx, qf);
#pragma unroll
      for (int i = 0; i < P; ++i) dqp[i] = make_float2(0.f, 0.f);
#pragma unroll
      for (int n = 0; n < N; ++n) {
        const float2 cf = coef[s * N + n];
        cvn[n] += cvp[s * N + n];
#pragma unroll
        for (int i = 0; i < P; ++i) {
          acc[n][i] = __ffma2_rn(f2(cf.x), gf[i], acc[n][i]);
          acc[n][i] = __ffma2_rn(f2(cf.y), qf[i], acc[n][i]);
          dqp[i] = __ffma2_rn(f2(cf.y), vf[n][i], dqp[i]);
        }
      }
      if (act) {
        float2* dq2 = reinterpret_cast<float2*>(dqs + (size_t)s * rc * VEC + (size_t)tid * VEC);
#pragma unroll
        for (int i = 0; i < P; ++i) {
          const float2 o = dq2[i];
          dq2[i] = make_float2(o.x + dqp[i].x, o.y + dqp[i].y);
        }
      }
    }
    if (act) {
#pragma unroll
      for (int n = 0; n < N; ++n) {
        float2 o[P];
#pragma unroll
        for (int i = 0; i < P; ++i) o[i] = __ffma2_rn(f2(cvn[n]), vf[n][i], acc[n][i]);
        reinterpret_cast<uint4*>(dv + ((size_t)n * BT + tok) * D)[tid] = pack2<T>(o);
      }
    }
  }
  if (act) {
    float* prow = dq_partial + (size_t)blockIdx.x * S * D;
    for (int s = 0; s < S; ++s) {
      const float4* src =
          reinterpret_cast<const float4*>(dqs + (size_t)s * rc * VEC + (size_t)tid * VEC);
      float4* dst = reinterpret_cast<float4*>(prow + (size_t)s * D + (size_t)tid * VEC);
#pragma unroll
      for (int i = 0; i < VEC / 4; ++i) dst[i] = src[i];
    }
  }
}

template <typename T, int N>
static cudaError_t launch_reg_bat_bwd_n(long long BT, int D, int S, int rc, const void* v,
                                        const void* q, const void* g, void* dv, float* dqp, int P,
                                        float eps, int variant, cudaStream_t st) {
  if (variant == kRegBwdStaged)
    return launch_smem(reg_bat_bwd_staged_kernel<T, N>, P, kGenericThreads,
                       reg_bwd_staged_total(N, S, rc, Dt<T>::kVec), st, static_cast<const T*>(v),
                       static_cast<const T*>(q), static_cast<const T*>(g), static_cast<T*>(dv),
                       dqp, BT, D, S, rc, eps);
  const size_t smem = reg_bwd_batched_layout(N, S, rc, Dt<T>::kVec).total;
  if (variant == 2)
    return launch_smem(reg_bat_bwd_kernel<T, N, 2>, P, kGenericThreads, smem, st,
                       static_cast<const T*>(v), static_cast<const T*>(q), static_cast<const T*>(g),
                       static_cast<T*>(dv), dqp, BT, D, S, rc, eps);
  return launch_smem(reg_bat_bwd_kernel<T, N, 1>, P, kGenericThreads, smem, st,
                     static_cast<const T*>(v), static_cast<const T*>(q), static_cast<const T*>(g),
                     static_cast<T*>(dv), dqp, BT, D, S, rc, eps);
}

template <typename T>
static cudaError_t launch_reg_bat_bwd_t(int N, long long BT, int D, int S, int rc, const void* v,
                                        const void* q, const void* g, void* dv, float* dqp, int P,
                                        float eps, int variant, cudaStream_t st) {
  switch (N) {
#define SY_RB_CASE(k) \
  case k:             \
    return launch_reg_bat_bwd_n<T, k>(BT, D, S, rc, v, q, g, dv, dqp, P, eps, variant, st);
    SY_RB_CASE(1) SY_RB_CASE(2) SY_RB_CASE(3) SY_RB_CASE(4) SY_RB_CASE(5) SY_RB_CASE(6)
    SY_RB_CASE(7) SY_RB_CASE(8) SY_RB_CASE(9)
#undef SY_RB_CASE
    default:
      return cudaErrorInvalidValue;
  }
}

// Which register-tile kernel takes a shape (rows of whole 16-byte chunks, at
// most one chunk per thread, N <= kBwdRegMaxN, S <= 16): the staged kernel where
// its shared memory (two buffers of the token's g chunks beside the half-pass
// kernel's) fits and S >= SY_TUNE_BWD_STAGED_MIN_S, else the half-pass kernel
// at two CTAs per SM where two fit the SM's shared memory (the per-block
// opt-in limit plus the 1 KiB the runtime reserves per block), else at one;
// 0 when none takes it.
int reg_bwd_batched_variant(int N, int D, int S, int dtype, int max_smem) {
  const int es = dtype == SY_F32 ? 4 : 2;
  if (N < 1 || N > kBwdRegMaxN || S < 1 || S > kBwdBatchedMaxS || (D * es) % 16) return 0;
  const int rc = D * es / 16;
  if (rc > kGenericThreads) return 0;
  if (S >= SY_TUNE_BWD_STAGED_MIN_S && reg_bwd_staged_total(N, S, rc, 16 / es) <= (size_t)max_smem)
    return kRegBwdStaged;
  const size_t smem = reg_bwd_batched_layout(N, S, rc, 16 / es).total;
  if (smem > (size_t)max_smem) return 0;
  return 2 * (smem + 1024) <= (size_t)max_smem + 1024 ? 2 : 1;
}

bool reg_bwd_batched_fits(int N, int D, int S, int dtype, int max_smem) {
  return reg_bwd_batched_variant(N, D, S, dtype, max_smem) > 0;
}

// CTAs of the chosen register-tile kernel resident per SM (0: none takes the shape).
int reg_bwd_batched_ctas_per_sm(int N, int D, int S, int dtype, int max_smem) {
  const int var = reg_bwd_batched_variant(N, D, S, dtype, max_smem);
  return var == 2 ? 2 : (var > 0 ? 1 : 0);
}

cudaError_t launch_reg_bwd_batched(long long BT, int N, int D, int S, int dtype, const void* v,
                                   const void* q, const void* g, void* dv, float* dq_partial,
                                   int P, float eps, int variant, cudaStream_t st) {
  const int rc = D * (dtype == SY_F32 ? 4 : 2) / 16;
  switch (dtype) {
    case SY_BF16:
      return launch_reg_bat_bwd_t<__nv_bfloat16>(N, BT, D, S, rc, v, q, g, dv, dq_partial, P, eps,
                                                 variant, st);
    case SY_F16:
      return launch_reg_bat_bwd_t<__half>(N, BT, D, S, rc, v, q, g, dv, dq_partial, P, eps,
                                          variant, st);
    case SY_F32:
      return launch_reg_bat_bwd_t<float>(N, BT, D, S, rc, v, q, g, dv, dq_partial, P, eps,
                                         variant, st);
    default:
      return cudaErrorInvalidValue;
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
                 long long R, int D, int normalize, int vec16) {
  constexpr int P = Dt<T>::kVec / 2;
  const int rc = vec16 ? D / Dt<T>::kVec : 0;
  for (long long row = blockIdx.x; row < R; row += gridDim.x) {
    const size_t base = (size_t)row * D;
    // the rows' first chunks are requested before the statistics are used,
    // so the two loads overlap instead of running back to back
    const int k0 = threadIdx.x;
    uint4 xa = make_uint4(0u, 0u, 0u, 0u), xb = xa;
    if (k0 < rc) {
      xa = reinterpret_cast<const uint4*>(o1 + base)[k0];
      xb = reinterpret_cast<const uint4*>(o2 + base)[k0];
    }
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
    if (vec16) {  // rows of whole 16-byte chunks, 16-byte aligned
      uint4* c4 = reinterpret_cast<uint4*>(o + base);
      for (int k = k0; k < rc; k += kGenericThreads) {
        if (k != k0) {
          xa = reinterpret_cast<const uint4*>(o1 + base)[k];
          xb = reinterpret_cast<const uint4*>(o2 + base)[k];
        }
        float2 x[P], y[P];
        unpack2<T>(xa, x);
        unpack2<T>(xb, y);
#pragma unroll
        for (int i = 0; i < P; ++i) x[i] = __ffma2_rn(x[i], f2(c1), __fmul2_rn(y[i], f2(c2)));
        c4[k] = pack2<T>(x);
      }
    } else {
      for (int d = threadIdx.x; d < D; d += kGenericThreads)
        o[base + d] = Dt<T>::from_f(
            fmaf(Dt<T>::to_f(o1[base + d]), c1, Dt<T>::to_f(o2[base + d]) * c2));
    }
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
                         int vec16, int grid, cudaStream_t st) {
  SY_BB_DTYPE_SWITCH(dtype, T,
                     return launch_smem(merge_kernel<T>, grid, kGenericThreads, 0, st,
                                        static_cast<const T*>(o1), ms1,
                                        static_cast<const T*>(o2), ms2, static_cast<T*>(o), ms, R,
                                        D, normalize, vec16))
}

}  // namespace sy
