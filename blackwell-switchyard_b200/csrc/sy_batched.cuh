// sy_batched.cuh -- batched-query forward on the register tile.
//
// block_attn_res_batched (src/switchyard/triton_op.py:438-501) evaluates S
// queries against the same sources: out[s] = sum_n softmax_n(q_s . k_n) v_n
// with k_n = v_n * rsqrt(mean(v_n^2) + eps). Here each token's N rows are read
// from HBM once (cp.async.bulk into a per-group ring, as in the register-tile
// forward) and held in registers as fp32; the queries (S rows of D, v's dtype)
// are copied into shared memory once per CTA. Per token a group of TG threads
// (thread t owns 16-byte chunks t, t+TG, ... of every row):
//
//   * sums of squares of the N rows -> reduce-scatter over the warp, fixed-order
//     sum over the group's warps through shared memory -> r_n, kept by lane n;
//   * queries in blocks of QB (as many as fill a 32-value reduce-scatter: 3 at
//     N = 9): dot_{s,n} = q_s . v_n from the registers (packed fp32 FMA), one
//     reduction for the whole block, a softmax per query over its N lanes
//     (segmented shuffles), alpha published to the warp's own shared slot as
//     fp32 pairs, and out[s] = sum_n alpha_{s,n} v_n written with one 16-byte
//     store per chunk.
//
// HBM traffic is the minimum ((N + S) rows per token); the work per token grows
// with S, so large S is bound by FP32 issue rather than bandwidth.
#pragma once

#include "sy_reg.cuh"

namespace sy {

constexpr int kBatchedMaxS = 16;
#ifndef SY_TUNE_BATCHED_TILE
#define SY_TUNE_BATCHED_TILE 144
#endif
#ifndef SY_TUNE_BATCHED_THREADS
#define SY_TUNE_BATCHED_THREADS 256
#endif
constexpr int kBatchedTileFloats = SY_TUNE_BATCHED_TILE;  // fp32 tile per thread (N * CPT * VEC)
constexpr int kBatchedThreads = SY_TUNE_BATCHED_THREADS;   // per CTA

// Shared memory beyond the tile layout: the S query rows.
__host__ __device__ inline size_t batched_q_off(const TileCfg& c) {
  return (tile_smem_layout(c).total + 127) / 128 * 128;
}

template <typename T, int N, int CPT>
__global__ void __launch_bounds__(kBatchedThreads, 1)
    reg_batched_kernel(const T* __restrict__ v, const T* __restrict__ q, T* __restrict__ out,
                       const TileCfg c, int S) {
  constexpr int VEC = Dt<T>::kVec;
  constexpr int P = VEC / 2;
  constexpr int M = 16;  // N <= 16 values per sum-of-squares reduction
  // queries per reduction round: as many as fill the 32 values of one
  // reduce-scatter (3 at N = 9), at most 4
  constexpr int QB = (32 / N) < 1 ? 1 : ((32 / N) > 4 ? 4 : (32 / N));
  static_assert(N * CPT * VEC <= kBatchedTileFloats, "tile does not fit the register budget");
  const TileSmem L = tile_smem_layout(c);
  unsigned char* stage0 = sy_smem + L.stages_off;
  float* red_base = reinterpret_cast<float*>(sy_smem + L.red_off);
  float* coef_base = reinterpret_cast<float*>(sy_smem + L.coef_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(sy_smem + L.bar_off);
  unsigned char* qsm = sy_smem + batched_q_off(c);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int grid = gridDim.x;
  const int cta = blockIdx.x;
  const int ntok = (cta < c.BT) ? (int)((c.BT - 1 - cta) / grid) + 1 : 0;
  const int wpg = c.tg >> 5;
  const int nwc = c.groups * wpg;

  if (c.N != N || c.groups < 1 || c.stages < c.groups || c.red_stride < 32 ||
      c.coef_stride < 2 * QB * N || S < 1 || S > kBatchedMaxS) {
    if (tid == 0) record_device_error(kDevErrBadPlan);
    return;
  }
  if (tid == 0) {
    for (int s = 0; s < c.stages; ++s) mbar_init(&full[s], 1);
    mbar_fence_init();
  }
  // the queries, once per CTA (S rows of row_bytes)
  {
    const uint4* src = reinterpret_cast<const uint4*>(q);
    uint4* dst = reinterpret_cast<uint4*>(qsm);
    const int total = S * c.row_chunks;
    for (int i = tid; i < total; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();

  const int g = tid / c.tg;
  const int tig = tid - g * c.tg;
  const int cw = tid >> 5;
  const int cw0 = g * wpg;
  const GroupRing ring = group_ring(c.stages, c.groups, g);
  const int ntok_g = ntok > g ? (ntok - 1 - g) / c.groups + 1 : 0;
  const uint64_t pol = policy_evict_first();
  const size_t nstride = (size_t)c.BT * c.row_bytes;
  const unsigned char* vb = reinterpret_cast<const unsigned char*>(v);

  if (tig == 0)
    for (int j = 0; j < ring.cnt && j < ntok_g; ++j)
      issue_token(stage0 + (size_t)(ring.base + j) * c.stage_bytes, &full[ring.base + j], vb,
                  cta + (long long)(g + j * c.groups) * grid, N, c.row_bytes, nstride, nullptr,
                  nullptr, 0, pol);

  bool cv[CPT];
#pragma unroll
  for (int cc = 0; cc < CPT; ++cc) cv[cc] = tig + cc * c.tg < c.row_chunks;
  const float inv_d = 1.f / (float)c.D;
  float4* alpha_slot = reinterpret_cast<float4*>(coef_base + (size_t)cw * c.coef_stride);

  // Sum M per-lane values over the group: reduce-scatter in the warp, then
  // the group's warps in order through shared memory. Every lane returns the
  // total of value lane >> 1 (lane, for the 32-value form). `k` counts the
  // reductions (buffer parity).
  int k = 0;
  auto group_reduce = [&](float (&a)[M]) {
    const float tl = warp_reduce_scatter<M>(a, lane);
    float* red = red_base + (size_t)(k & 1) * nwc * c.red_stride;
    ++k;
    if ((lane & 1) == 0) red[cw * c.red_stride + (lane >> 1)] = tl;
    if (wpg > 1)
      named_sync(1 + g, c.tg);
    else
      __syncwarp();
    float tot = 0.f;
    for (int w = 0; w < wpg; ++w) tot += red[(cw0 + w) * c.red_stride + (lane >> 1)];
    return tot;
  };
  auto group_reduce32 = [&](float (&a)[32]) {
    const float tl = warp_reduce_scatter<32>(a, lane);
    float* red = red_base + (size_t)(k & 1) * nwc * c.red_stride;
    ++k;
    red[cw * c.red_stride + lane] = tl;
    if (wpg > 1)
      named_sync(1 + g, c.tg);
    else
      __syncwarp();
    float tot = 0.f;
    for (int w = 0; w < wpg; ++w) tot += red[(cw0 + w) * c.red_stride + lane];
    return tot;
  };

  int slot = 0;
  uint32_t ph = 0;
  for (int j = 0; j < ntok_g; ++j) {
    const int sidx = ring.base + slot;
    if (!mbar_wait(&full[sidx], ph)) return;
    const unsigned char* tile = stage0 + (size_t)sidx * c.stage_bytes;
    const long long tok = cta + (long long)(g + j * c.groups) * grid;

    Tile<T, N, CPT, false> x;
#pragma unroll
    for (int n = 0; n < N; ++n)
#pragma unroll
      for (int cc = 0; cc < CPT; ++cc)
        x.load(n, cc, cv[cc] ? lds128(tile + (size_t)n * c.row_bytes + (tig + cc * c.tg) * 16)
                             : make_uint4(0u, 0u, 0u, 0u));

    // ---- sums of squares -> r_n (lane n) ----
    float r_l;
    {
      float a[M];
#pragma unroll
      for (int i = 0; i < M; ++i) a[i] = 0.f;
#pragma unroll
      for (int n = 0; n < N; ++n) {
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int cc = 0; cc < CPT; ++cc) {
          float2 p[P];
          x.get(n, cc, p);
#pragma unroll
          for (int i = 0; i < P; ++i) acc = __ffma2_rn(p[i], p[i], acc);
        }
        a[n] = acc.x + acc.y;
      }
      const float tot = group_reduce(a);
      // every thread of the group has copied the stage: refill it
      if (tig == 0 && j + ring.cnt < ntok_g) {
        fence_proxy_async();
        issue_token(stage0 + (size_t)sidx * c.stage_bytes, &full[sidx], vb,
                    cta + (long long)(g + (j + ring.cnt) * c.groups) * grid, N, c.row_bytes,
                    nstride, nullptr, nullptr, 0, pol);
      }
      const int ln = lane < N ? lane : 0;
      r_l = rsqrtf(__shfl_sync(kFull, tot, 2 * ln) * inv_d + c.eps);
    }

    // ---- queries in blocks of QB, from the registers ----
    for (int s0 = 0; s0 < S; s0 += QB) {
      const int qb = S - s0 < QB ? S - s0 : QB;  // queries in this block (warp-uniform)
      // value qi*N + n = q_{s0+qi} . v_n (this thread's part)
      float a[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) a[i] = 0.f;
#pragma unroll
      for (int qi = 0; qi < QB; ++qi) {
        if (qi < qb) {
          float2 acc[N];
#pragma unroll
          for (int n = 0; n < N; ++n) acc[n] = make_float2(0.f, 0.f);
#pragma unroll
          for (int cc = 0; cc < CPT; ++cc) {
            float2 qf[P];
            unpack2<T>(cv[cc] ? lds128(qsm + (size_t)(s0 + qi) * c.row_bytes +
                                       (tig + cc * c.tg) * 16)
                              : make_uint4(0u, 0u, 0u, 0u),
                       qf);
#pragma unroll
            for (int n = 0; n < N; ++n) {
              float2 p[P];
              x.get(n, cc, p);
#pragma unroll
              for (int i = 0; i < P; ++i) acc[n] = __ffma2_rn(qf[i], p[i], acc[n]);
            }
          }
#pragma unroll
          for (int n = 0; n < N; ++n) a[qi * N + n] = acc[n].x + acc[n].y;
        }
      }
      // lane L: the group total of value L
      const float tot = group_reduce32(a);
      // softmax over the N sources of each query: lanes qi*N .. qi*N+N-1
      const bool act = lane < qb * N;
      const int qi = act ? lane / N : 0;
      const int n = act ? lane - qi * N : 0;
      const int base = qi * N;
      // every lane takes part in each shuffle (full mask); selects come after
      const float r_n = __shfl_sync(kFull, r_l, n);
      const float logit = act ? tot * r_n : -INFINITY;
      float m = -INFINITY;
#pragma unroll
      for (int jj = 0; jj < N; ++jj) m = fmaxf(m, __shfl_sync(kFull, logit, base + jj));
      const float e = act ? expf(logit - m) : 0.f;
      float l = 0.f;
#pragma unroll
      for (int jj = 0; jj < N; ++jj) l += __shfl_sync(kFull, e, base + jj);
      const float al = c.raw ? e : e / l;
      if (c.mstats != nullptr && act && n == 0)
        reinterpret_cast<float2*>(c.mstats)[(size_t)(s0 + qi) * c.BT + tok] = make_float2(m, l);
      __syncwarp();  // the previous block's reads of the slot are done
      if (act) reinterpret_cast<float2*>(alpha_slot)[lane] = make_float2(al, al);
      __syncwarp();
#pragma unroll
      for (int qo = 0; qo < QB; ++qo) {
        if (qo < qb) {
          float2 alp[N];
#pragma unroll
          for (int k2 = 0; k2 < N; ++k2) alp[k2] = reinterpret_cast<const float2*>(alpha_slot)[qo * N + k2];
          T* orow = out + ((size_t)(s0 + qo) * c.BT + tok) * c.D;
#pragma unroll
          for (int cc = 0; cc < CPT; ++cc) {
            if (!cv[cc]) continue;
            float2 o[P];
#pragma unroll
            for (int i = 0; i < P; ++i) o[i] = make_float2(0.f, 0.f);
#pragma unroll
            for (int k2 = 0; k2 < N; ++k2) {
              float2 p[P];
              x.get(k2, cc, p);
#pragma unroll
              for (int i = 0; i < P; ++i) o[i] = __ffma2_rn(alp[k2], p[i], o[i]);
            }
            stg128(orow + (size_t)(tig + cc * c.tg) * VEC, pack2<T>(o));
          }
        }
      }
    }

    if (++slot == ring.cnt) {
      slot = 0;
      ph ^= 1u;
    }
  }
}

template <typename T, int N>
cudaError_t launch_batched_n(const TileCfg& c, int grid, int cpt, int S, const void* v,
                             const void* q, void* out, cudaStream_t st) {
  const size_t smem = batched_q_off(c) + (size_t)S * c.row_bytes;
  const dim3 block(c.groups * c.tg);
  if ((int)block.x > kBatchedThreads) return cudaErrorInvalidConfiguration;
  const T* vp = static_cast<const T*>(v);
  const T* qp = static_cast<const T*>(q);
  T* op = static_cast<T*>(out);
  constexpr int VEC = Dt<T>::kVec;
  if constexpr (N * 1 * VEC <= kBatchedTileFloats)
    if (cpt == 1)
      return launch_smem(reg_batched_kernel<T, N, 1>, grid, block, smem, st, vp, qp, op, c, S);
  if constexpr (N * 2 * VEC <= kBatchedTileFloats)
    if (cpt == 2)
      return launch_smem(reg_batched_kernel<T, N, 2>, grid, block, smem, st, vp, qp, op, c, S);
  if constexpr (N * 4 * VEC <= kBatchedTileFloats)
    if (cpt == 4)
      return launch_smem(reg_batched_kernel<T, N, 4>, grid, block, smem, st, vp, qp, op, c, S);
  return cudaErrorInvalidValue;
}

template <typename T>
cudaError_t launch_batched_t(const TileCfg& c, int grid, int cpt, int S, const void* v,
                             const void* q, void* out, cudaStream_t st) {
  switch (c.N) {
    SY_REG_CASES(launch_batched_n, c, grid, cpt, S, v, q, out, st)
    default:
      return cudaErrorInvalidValue;
  }
}

// Per-dtype entry points (sy_batched_{bf16,f16,f32}.cu).
#define SY_BATCHED_DECL(dt)                                                                   \
  cudaError_t launch_batched_##dt(const TileCfg& c, int grid, int cpt, int S, const void* v, \
                                  const void* q, void* out, cudaStream_t st);
SY_BATCHED_DECL(bf16)
SY_BATCHED_DECL(f16)
SY_BATCHED_DECL(f32)
#undef SY_BATCHED_DECL

}  // namespace sy
