// sy_batched.cuh -- batched-query forward on the register tile.
//
// block_attn_res_batched (src/switchyard/triton_op.py:438-501) evaluates S
// queries against the same sources: out[s] = sum_n softmax_n(q_s . k_n) v_n
// with k_n = v_n * rsqrt(mean(v_n^2) + eps). Here each token's N rows are read
// from HBM once (cp.async.bulk into a per-group ring, as in the register-tile
// forward) and held in registers as fp32; the queries (S rows of D, v's dtype)
// are copied into shared memory once per CTA, padded with zero rows to SB = 4, 8
// or 16 slots so that every query loop is unrolled at compile time. Per token a
// group of TG threads (thread t owns 16-byte chunks t, t+TG, ... of every row):
//
//   * the S x N dots q_s . v_n from the registers (packed fp32 FMA), QB queries
//     at a time (as many as fill a 32-value reduce-scatter: 3 at N = 9), and
//     the N sums of squares in the spare lanes of the last block (or a block of
//     their own): one warp reduce-scatter per block, all issued back to back;
//   * one exchange across the group's warps for the whole token -- the
//     blocks' warp totals through shared memory, one named barrier, then every
//     warp adds them in warp order -- after which the stage is refilled;
//   * per query block a softmax over its N lanes (segmented shuffles), alpha
//     published to the warp's own shared slot as fp32 pairs, index s * N + n;
//   * out[s] = sum_n alpha_{s,n} v_n for every query from the registers, one
//     16-byte store per chunk.
//
// HBM traffic is the minimum ((N + S) rows per token); the FMA work per token
// grows with S, so large S is bound by FP32 issue rather than bandwidth. The
// single barrier matters: every warp of a group reaches the chain of
// reductions, barrier and softmax at the same time, and that chain, not the
// FMA count, sets the pace (one barrier and softmax pass per query block
// before).
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

// Query slots for S queries (the padded count the kernel is compiled for).
__host__ __device__ constexpr int batched_slots(int S) { return S <= 4 ? 4 : (S <= 8 ? 8 : 16); }
// Queries per 32-value reduction block at N sources (at most 4).
__host__ __device__ constexpr int batched_qb(int N) {
  return (32 / N) < 1 ? 1 : ((32 / N) > 4 ? 4 : (32 / N));
}
// Reduction blocks per token: the query blocks, plus one for the sums of
// squares unless they fit the last query block's spare lanes.
__host__ __device__ constexpr int batched_blocks(int N, int SB) {
  return (SB + batched_qb(N) - 1) / batched_qb(N) +
         ((SB - ((SB + batched_qb(N) - 1) / batched_qb(N) - 1) * batched_qb(N)) * N + N <= 32
              ? 0
              : 1);
}
// Per-warp scratch in floats: the blocks' warp totals (one reduction buffer)
// and the alpha pairs of all query slots (16-byte multiple).
__host__ __device__ constexpr int batched_red_stride(int N, int S) {
  return 32 * batched_blocks(N, batched_slots(S));
}
__host__ __device__ constexpr int batched_coef_stride(int N, int S) {
  return (2 * batched_slots(S) * N + 3) / 4 * 4;
}

// Shared memory beyond the tile layout: the query slots.
__host__ __device__ inline size_t batched_q_off(const TileCfg& c) {
  return (tile_smem_layout(c).total + 127) / 128 * 128;
}

template <typename T, int N, int CPT, int SB>
__global__ void __launch_bounds__(kBatchedThreads, 1)
    reg_batched_kernel(const T* __restrict__ v, const T* __restrict__ q, T* __restrict__ out,
                       const TileCfg c, int S) {
  constexpr int VEC = Dt<T>::kVec;
  constexpr int P = VEC / 2;
  constexpr int QB = batched_qb(N);
  constexpr int NBQ = (SB + QB - 1) / QB;  // query blocks
  constexpr int NB = batched_blocks(N, SB);
  constexpr int SS_BLOCK = NB - 1;  // block holding the sums of squares
  constexpr int SS_BASE = NB > NBQ ? 0 : (SB - (NBQ - 1) * QB) * N;  // and their first lane
  static_assert(N * CPT * VEC <= kBatchedTileFloats, "tile does not fit the register budget");
  static_assert(SS_BASE + N <= 32, "sums of squares must fit one block");
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

  if (c.N != N || c.groups < 1 || c.stages < c.groups || c.red_stride < 32 * NB ||
      c.coef_stride < 2 * SB * N || S < 1 || S > SB) {
    if (tid == 0) record_device_error(kDevErrBadPlan);
    return;
  }
  if (tid == 0) {
    for (int s = 0; s < c.stages; ++s) mbar_init(&full[s], 1);
    mbar_fence_init();
  }
  // the queries, once per CTA (S rows of row_bytes), then zero rows up to SB
  {
    const uint4* src = reinterpret_cast<const uint4*>(q);
    uint4* dst = reinterpret_cast<uint4*>(qsm);
    const int given = S * c.row_chunks;
    const int total = SB * c.row_chunks;
    for (int i = tid; i < total; i += blockDim.x)
      dst[i] = i < given ? src[i] : make_uint4(0u, 0u, 0u, 0u);
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
  float2* alpha_slot = reinterpret_cast<float2*>(coef_base + (size_t)cw * c.coef_stride);

  int k = 0;  // tokens done by this group (reduction buffer parity)
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

    // ---- every block's partial dots (and the sums of squares), reduced over
    // the warp back to back: lane L then holds the warp total of value L ----
    // (query slots s >= S are zero rows: their work is skipped, uniformly)
    float t[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      t[b] = 0.f;
      if (b != SS_BLOCK && b * QB >= S) continue;
      float a[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) a[i] = 0.f;
#pragma unroll
      for (int qi = 0; qi < QB; ++qi) {
        const int s = b * QB + qi;
        if (b < NBQ && s < SB && s < S) {
          float2 acc[N];
#pragma unroll
          for (int n = 0; n < N; ++n) acc[n] = make_float2(0.f, 0.f);
#pragma unroll
          for (int cc = 0; cc < CPT; ++cc) {
            // lanes past the row's last chunk (short rows) read nothing
            float2 qf[P];
            unpack2<T>(cv[cc] ? lds128(qsm + (size_t)s * c.row_bytes + (tig + cc * c.tg) * 16)
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
      if (b == SS_BLOCK) {
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
          a[SS_BASE + n] = acc.x + acc.y;
        }
      }
      t[b] = warp_reduce_scatter<32>(a, lane);
    }

    // ---- one exchange across the group's warps ----
    {
      float* red = red_base + (size_t)(k & 1) * nwc * c.red_stride;
#pragma unroll
      for (int b = 0; b < NB; ++b) red[cw * c.red_stride + b * 32 + lane] = t[b];
      if (wpg > 1)
        named_sync(1 + g, c.tg);
      else
        __syncwarp();
      // every thread of the group has copied the stage: refill it
      if (tig == 0 && j + ring.cnt < ntok_g) {
        fence_proxy_async();
        issue_token(stage0 + (size_t)sidx * c.stage_bytes, &full[sidx], vb,
                    cta + (long long)(g + (j + ring.cnt) * c.groups) * grid, N, c.row_bytes,
                    nstride, nullptr, nullptr, 0, pol);
      }
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        float tot = 0.f;
        for (int w = 0; w < wpg; ++w) tot += red[(cw0 + w) * c.red_stride + b * 32 + lane];
        t[b] = tot;
      }
      ++k;
    }
    const int ln = lane < N ? lane : 0;
    const float r_l = rsqrtf(__shfl_sync(kFull, t[SS_BLOCK], SS_BASE + ln) * inv_d + c.eps);

    // ---- softmax per query block: lanes qi*N .. qi*N+N-1 hold query qi's logits ----
    __syncwarp();  // the previous token's reads of the alpha slot are done
#pragma unroll
    for (int b = 0; b < NBQ; ++b) {
      if (b * QB >= S) break;
      const int qb = SB - b * QB < QB ? SB - b * QB : QB;  // compile-time after unrolling
      const bool act = lane < qb * N;
      const int qi = act ? lane / N : 0;
      const int n = act ? lane - qi * N : 0;
      const int base = qi * N;
      // every lane takes part in each shuffle (full mask); selects come after
      const float r_n = __shfl_sync(kFull, r_l, n);
      const float logit = act ? t[b] * r_n : -INFINITY;
      float m = -INFINITY;
#pragma unroll
      for (int jj = 0; jj < N; ++jj) m = fmaxf(m, __shfl_sync(kFull, logit, base + jj));
      const float e = act ? expf(logit - m) : 0.f;
      float l = 0.f;
#pragma unroll
      for (int jj = 0; jj < N; ++jj) l += __shfl_sync(kFull, e, base + jj);
      const float al = c.raw ? e : e / l;
      const int s = b * QB + qi;
      if (c.mstats != nullptr && act && n == 0 && s < S)
        reinterpret_cast<float2*>(c.mstats)[(size_t)s * c.BT + tok] = make_float2(m, l);
      if (act) alpha_slot[b * QB * N + lane] = make_float2(al, al);
    }
    __syncwarp();

    // ---- out[s] = sum_n alpha_{s,n} v_n ----
#pragma unroll
    for (int s = 0; s < SB; ++s) {
      if (s < S) {
        float2 alp[N];
#pragma unroll
        for (int n = 0; n < N; ++n) alp[n] = alpha_slot[s * N + n];
        T* orow = out + ((size_t)s * c.BT + tok) * c.D;
#pragma unroll
        for (int cc = 0; cc < CPT; ++cc) {
          if (!cv[cc]) continue;
          float2 o[P];
#pragma unroll
          for (int i = 0; i < P; ++i) o[i] = make_float2(0.f, 0.f);
#pragma unroll
          for (int n = 0; n < N; ++n) {
            float2 p[P];
            x.get(n, cc, p);
#pragma unroll
            for (int i = 0; i < P; ++i) o[i] = __ffma2_rn(alp[n], p[i], o[i]);
          }
          stg128(orow + (size_t)(tig + cc * c.tg) * VEC, pack2<T>(o));
        }
      }
    }

    if (++slot == ring.cnt) {
      slot = 0;
      ph ^= 1u;
    }
  }
}

template <typename T, int N, int SB>
cudaError_t launch_batched_ns(const TileCfg& c, int grid, int cpt, int S, const void* v,
                              const void* q, void* out, cudaStream_t st) {
  const size_t smem = batched_q_off(c) + (size_t)SB * c.row_bytes;
  const dim3 block(c.groups * c.tg);
  if ((int)block.x > kBatchedThreads) return cudaErrorInvalidConfiguration;
  const T* vp = static_cast<const T*>(v);
  const T* qp = static_cast<const T*>(q);
  T* op = static_cast<T*>(out);
  constexpr int VEC = Dt<T>::kVec;
  if constexpr (N * 1 * VEC <= kBatchedTileFloats)
    if (cpt == 1)
      return launch_smem(reg_batched_kernel<T, N, 1, SB>, grid, block, smem, st, vp, qp, op, c, S);
  if constexpr (N * 2 * VEC <= kBatchedTileFloats)
    if (cpt == 2)
      return launch_smem(reg_batched_kernel<T, N, 2, SB>, grid, block, smem, st, vp, qp, op, c, S);
  if constexpr (N * 4 * VEC <= kBatchedTileFloats)
    if (cpt == 4)
      return launch_smem(reg_batched_kernel<T, N, 4, SB>, grid, block, smem, st, vp, qp, op, c, S);
  return cudaErrorInvalidValue;
}

template <typename T, int N>
cudaError_t launch_batched_n(const TileCfg& c, int grid, int cpt, int S, const void* v,
                             const void* q, void* out, cudaStream_t st) {
  switch (batched_slots(S)) {
    case 4:
      return launch_batched_ns<T, N, 4>(c, grid, cpt, S, v, q, out, st);
    case 8:
      return launch_batched_ns<T, N, 8>(c, grid, cpt, S, v, q, out, st);
    default:
      return launch_batched_ns<T, N, 16>(c, grid, cpt, S, v, q, out, st);
  }
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
