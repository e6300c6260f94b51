// sy_stream_bwd.cuh -- "row stream" backward for rows of 4 KiB and more.
//
// The register-tile backward holds a token's N source rows in registers; at
// 16 KiB rows (D = 8192 bf16) or N > 16 they no longer fit. Here K warps share
// each token (K = 1 .. 16), warp k owning chunks 32 CPL k .. 32 CPL (k+1) - 1 of
// every row (CPL = 1, 2 or 4 per lane: more warps per token for the same row
// keep fewer tokens in flight, see the planner),
// and the token's rows stream through the K warps' shared ring of R row
// buffers (cp.async.bulk, one mbarrier per buffer) in the order
//
//   g,  v_0 .. v_{N-1}  (pass A, from HBM),  v_0 .. v_{N-1}  (pass B, again)
//
// so a token is 2N + 1 rows of the stream. Pass A keeps g in registers as fp32
// and forms each warp's part of G_n = g . v_n (butterfly over the lanes); the
// K warps meet once per token at a named barrier and every warp adds the K
// parts in warp order, so all of them hold the bitwise-same G. The saved
// statistics give alpha_n = exp(logit_n - lse) and, with G,
//
//   S = sum_n alpha_n G_n,  dlogit_n = alpha_n (G_n - S),
//   da_n = dlogit_n r_n,    cv_n = -dlogit_n logit_n r_n^2 / D,
//
// held by lane n mod 32 (in its register slot n / 32: N <= 64, one slot per
// 32 sources). Pass B reads each row a second time -- the copy that pass A
// loaded with an evict-last hint, normally still in L2 -- and writes
//
//   dv_n = alpha_n g + da_n w + cv_n v_n,     dw += da_n v_n  (registers).
//
// A buffer is released by the last of the K warps to finish with it (a shared
// counter), which refills it with the row R ahead. At the end each CTA adds
// its token streams' dw in stream order into one fp32 partial row.
//
// Reference: the same two passes as the reference's tiled backward,
// src/switchyard/triton_op.py:280-330 (_bwd_stats: per-token alpha, da and the
// sum-of-squares coefficient) and :331-378 (_bwd_apply: dv and dw), with the
// derivation at :205-214; here both passes run in one kernel per token, from
// the forward's saved statistics instead of recomputed reductions.
#pragma once

#include "sy_stream.cuh"

namespace sy {

struct StreamBwdCfg {
  long long BT;
  int N, D;
  int row_chunks;  // 16-byte chunks per row: exactly 32 * cpl * kw
  int cpl;         // 16-byte chunks per lane and row: 1, 2 or 4
  int row_bytes;
  int kw;          // warps per token
  int warps;       // per CTA, a multiple of kw
  int ring;        // row buffers per token stream
  int stats_stride;
};

struct StreamBwdSmem {
  size_t w_off, ring_off, bar_off, xg_off, cnt_off, total;
};

// fp32 w (as planes of float4, like the forward), the streams' rings and full
// barriers, the per-token exchange of G parts ([streams][2][kw][64] floats,
// double-buffered by token parity; 32 per register slot) and the
// buffer-release counters.
__host__ __device__ inline StreamBwdSmem stream_bwd_smem_layout(const StreamBwdCfg& c) {
  const int kw = c.kw > 0 ? c.kw : 1;
  const size_t streams = (size_t)(c.warps / kw);
  StreamBwdSmem s;
  s.w_off = 0;
  s.ring_off = ((size_t)c.D * 4 + 127) / 128 * 128;
  s.bar_off = s.ring_off + streams * c.ring * c.row_bytes;
  s.xg_off = s.bar_off + streams * c.ring * 8;
  s.cnt_off = s.xg_off + streams * 2 * kw * 64 * 4;
  s.total = s.cnt_off + (streams * c.ring * 4 + 15) / 16 * 16;
  return s;
}

// 16 warps: g and the dw accumulators take 2 * 4 * 8 fp32 registers per lane,
// which leaves room under the 128-register cap of a 512-thread CTA.
#ifndef SY_TUNE_STREAM_BWD_WARPS
#define SY_TUNE_STREAM_BWD_WARPS 16
#endif
constexpr int kStreamBwdThreads = 32 * SY_TUNE_STREAM_BWD_WARPS;
constexpr int kStreamBwdMaxCpl = 4;  // 16-byte chunks per lane and row: 1, 2 or 4
constexpr int kStreamBwdMaxN = 64;    // lane n % 32, register slot n / 32, holds source n

// L2 hint for pass A's copy of a row (pass B reads it again).
#ifndef SY_TUNE_STREAM_BWD_KEEP
#define SY_TUNE_STREAM_BWD_KEEP 1  // 1: evict_last, 0: evict_first
#endif

// SL: register slots of per-source coefficients per lane (1: N <= 32, 2: N <= 64).
// CPL: 16-byte chunks per lane and row (a row is K warps x 32 lanes x CPL).
template <typename T, int SL, int CPL>
__global__ void __launch_bounds__(kStreamBwdThreads, 1)
    stream_bwd_kernel(const T* __restrict__ v, const void* __restrict__ w, int w_dtype,
                      const T* __restrict__ gin, const float* __restrict__ stats,
                      T* __restrict__ dv, float* __restrict__ dw_partial, const StreamBwdCfg c) {
  constexpr int VEC = Dt<T>::kVec;
  constexpr int P = VEC / 2;
  const StreamBwdSmem L = stream_bwd_smem_layout(c);
  float* wsm = reinterpret_cast<float*>(sy_smem + L.w_off);
  unsigned char* ring0 = sy_smem + L.ring_off;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sy_smem + L.bar_off);
  float* xg0 = reinterpret_cast<float*>(sy_smem + L.xg_off);
  int* cnt0 = reinterpret_cast<int*>(sy_smem + L.cnt_off);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int wi = tid >> 5;
  const int K = c.kw;
  const int RC = c.row_chunks;
  const int RB = c.row_bytes;
  if (K < 1 || K > 16 || c.warps % K != 0 || c.warps != (int)(blockDim.x >> 5) || c.ring < 2 ||
      c.cpl != CPL || RC != 32 * CPL * K || RB != 16 * RC || c.N < 1 || c.N > 32 * SL ||
      (K > 1 && c.warps / K > 15)) {
    if (tid == 0) record_device_error(kDevErrBadPlan);
    return;
  }
  const int streams = c.warps / K;
  if (tid == 0) {
    for (int i = 0; i < streams * c.ring; ++i) mbar_init(&bars[i], 1);
    mbar_fence_init();
  }
  for (int i = tid; i < streams * c.ring; i += blockDim.x) cnt0[i] = 0;
  pdl_wait();  // a programmatic dependent of the forward: inputs after it completes
  for (int d = tid; d < c.D; d += blockDim.x) {
    const int ch = d / VEC, e = d - ch * VEC;
    wsm[((e >> 2) * RC + ch) * 4 + (e & 3)] = load_any(w, w_dtype, d);
  }
  __syncthreads();

  const int N = c.N;
  const int gi = wi / K, wk = wi - gi * K;
  const long long tstride = (long long)gridDim.x * streams;
  const long long tok0 = blockIdx.x + (long long)gridDim.x * gi;
  const int ntok = tok0 < c.BT ? (int)((c.BT - 1 - tok0) / tstride) + 1 : 0;
  const int LT = 2 * N + 1;      // stream rows per token
  const int nrows = ntok * LT;   // the planner keeps this below 2^31
  unsigned char* ring = ring0 + (size_t)gi * c.ring * RB;
  uint64_t* bar = bars + gi * c.ring;
  float* xg = xg0 + (size_t)gi * 2 * K * 64;
  int* cnt = cnt0 + gi * c.ring;
  const size_t nstride = (size_t)c.BT * RB;
  const unsigned char* vb = reinterpret_cast<const unsigned char*>(v);
  const unsigned char* gb = reinterpret_cast<const unsigned char*>(gin);

  // stream row q: index i = q mod (2N + 1) of token q / (2N + 1)
  auto issue_row = [&](int slot_, int q) {
    if (q >= nrows) return;
    const int jj = q / LT, ii = q - jj * LT;
    const size_t toff = (size_t)(tok0 + tstride * jj) * RB;
    const unsigned char* src;
    uint64_t pol;
    if (ii == 0) {
      src = gb + toff;
      pol = policy_evict_first();
    } else if (ii <= N) {
      src = vb + (size_t)(ii - 1) * nstride + toff;
      pol = SY_TUNE_STREAM_BWD_KEEP ? policy_evict_last() : policy_evict_first();
    } else {
      src = vb + (size_t)(ii - 1 - N) * nstride + toff;
      pol = policy_evict_first();
    }
    mbar_arrive_expect_tx(&bar[slot_], (uint32_t)RB);
    bulk_g2s(ring + (size_t)slot_ * RB, src, (uint32_t)RB, &bar[slot_], pol);
  };
  // The last of the K warps to finish with a buffer refills it.
  auto release = [&](int slot_, int q) {
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      if (atomicAdd(&cnt[slot_], 1) == K - 1) {
        cnt[slot_] = 0;
        __threadfence_block();
        fence_proxy_async();
        issue_row(slot_, q + c.ring);
      }
    }
  };
  if (wk == 0 && lane == 0)
    for (int s = 0; s < c.ring; ++s) issue_row(s, s);

  const int cb = wk * (32 * CPL) + lane;  // this lane's chunks: cb + 32k
  const float inv_d = 1.f / (float)c.D;
  float2 dw2[CPL][P];
#pragma unroll
  for (int k = 0; k < CPL; ++k)
#pragma unroll
    for (int i = 0; i < P; ++i) dw2[k][i] = make_float2(0.f, 0.f);

  bool ok = true;
  int q = 0;
  int ring_slot = 0;        // slot and phase of stream row q (q mod R, (q / R) & 1)
  uint32_t ring_ph = 0;
  for (int j = 0; j < ntok && ok; ++j) {
    const long long tok = tok0 + tstride * j;
    // lane n % 32, slot n / 32: source n's saved logit and inverse RMS
    // (used after pass A)
    const float* st = stats + tok * c.stats_stride;
    float s_logit[SL], s_r[SL];
#pragma unroll
    for (int sl = 0; sl < SL; ++sl) {
      const int n = lane + 32 * sl;
      s_logit[sl] = n < N ? st[n] : 0.f;
      s_r[sl] = n < N ? st[N + n] : 0.f;
    }
    const float lse = st[2 * N + 1];

    // ---- g: to registers as fp32 ----
    float2 gf[CPL][P];
    {
      const int slot = ring_slot;
      const uint32_t ph = ring_ph;
      if (++ring_slot == c.ring) {
        ring_slot = 0;
        ring_ph ^= 1u;
      }
      if (!mbar_wait(&bar[slot], ph)) {
        ok = false;
        break;
      }
      const unsigned char* row = ring + (size_t)slot * RB;
#pragma unroll
      for (int k = 0; k < CPL; ++k) unpack2<T>(lds128(row + (cb + 32 * k) * 16), gf[k]);
      release(slot, q);
      ++q;
    }

    // ---- pass A: this warp's part of G_n = g . v_n, lane n % 32 keeps it ----
    float myg[SL];
#pragma unroll
    for (int sl = 0; sl < SL; ++sl) myg[sl] = 0.f;
    for (int n = 0; n < N; ++n, ++q) {
      const int slot = ring_slot;
      const uint32_t ph = ring_ph;
      if (++ring_slot == c.ring) {
        ring_slot = 0;
        ring_ph ^= 1u;
      }
      if (!mbar_wait(&bar[slot], ph)) {
        ok = false;
        break;
      }
      const unsigned char* row = ring + (size_t)slot * RB;
      float2 acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
      for (int k = 0; k < CPL; ++k) {
        float2 x[P];
        unpack2<T>(lds128(row + (cb + 32 * k) * 16), x);
#pragma unroll
        for (int i = 0; i < P; ++i) acc[i & 1] = __ffma2_rn(gf[k][i], x[i], acc[i & 1]);
      }
      release(slot, q);
      acc[0] = __fadd2_rn(acc[0], acc[1]);
      float s = acc[0].x + acc[0].y;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(kFull, s, off);
#pragma unroll
      for (int sl = 0; sl < SL; ++sl)
        if (n >> 5 == sl && lane == (n & 31)) myg[sl] = s;  // (the slot test is warp-uniform)
    }
    if (!ok) break;

    // ---- the K warps' parts of G, added in warp order by every warp ----
    float* xr = xg + (j & 1) * K * 64;
#pragma unroll
    for (int sl = 0; sl < SL; ++sl) xr[wk * 64 + 32 * sl + lane] = myg[sl];
    if (K > 1)
      named_sync(1 + gi, 32 * K);
    else
      __syncwarp();
    float G[SL];
#pragma unroll
    for (int sl = 0; sl < SL; ++sl) {
      G[sl] = xr[32 * sl + lane];
      for (int k2 = 1; k2 < K; ++k2) G[sl] += xr[k2 * 64 + 32 * sl + lane];
    }

    // ---- coefficients: lane n % 32, slot n / 32, owns source n ----
    float alpha[SL], da_l[SL], cv_l[SL];
    float ag = 0.f;
#pragma unroll
    for (int sl = 0; sl < SL; ++sl) {
      alpha[sl] = lane + 32 * sl < N ? expf(s_logit[sl] - lse) : 0.f;
      ag = sl == 0 ? alpha[0] * G[0] : fmaf(alpha[sl], G[sl], ag);
    }
    const float S = warp_sum(ag);
#pragma unroll
    for (int sl = 0; sl < SL; ++sl) {
      const float dl = alpha[sl] * (G[sl] - S);
      da_l[sl] = dl * s_r[sl];
      cv_l[sl] = -dl * s_logit[sl] * s_r[sl] * s_r[sl] * inv_d;
    }

    // ---- pass B: dv_n = alpha_n g + da_n w + cv_n v_n ; dw += da_n v_n ----
    T* dtok = dv + (size_t)tok * c.D + (size_t)cb * VEC;
    for (int n = 0; n < N; ++n, ++q) {
      // source n's coefficients from lane n % 32, slot n / 32 (warp-uniform)
      float a_src = alpha[0], d_src = da_l[0], c_src = cv_l[0];
#pragma unroll
      for (int sl = 1; sl < SL; ++sl)
        if (n >> 5 == sl) a_src = alpha[sl], d_src = da_l[sl], c_src = cv_l[sl];
      const float ka = __shfl_sync(kFull, a_src, n & 31);
      const float kd = __shfl_sync(kFull, d_src, n & 31);
      const float kc = __shfl_sync(kFull, c_src, n & 31);
      const int slot = ring_slot;
      const uint32_t ph = ring_ph;
      if (++ring_slot == c.ring) {
        ring_slot = 0;
        ring_ph ^= 1u;
      }
      if (!mbar_wait(&bar[slot], ph)) {
        ok = false;
        break;
      }
      const unsigned char* row = ring + (size_t)slot * RB;
      T* drow = dtok + (size_t)n * c.BT * c.D;
#pragma unroll
      for (int k = 0; k < CPL; ++k) {
        float2 x[P], d[P];
        unpack2<T>(lds128(row + (cb + 32 * k) * 16), x);
        const float4* wp = reinterpret_cast<const float4*>(wsm) + (cb + 32 * k);
#pragma unroll
        for (int i = 0; i < P; i += 2) {
          const float4 wv = wp[(i / 2) * RC];
          const float2 w0 = make_float2(wv.x, wv.y), w1 = make_float2(wv.z, wv.w);
          d[i] = __ffma2_rn(f2(kc), x[i], __ffma2_rn(f2(kd), w0, __fmul2_rn(f2(ka), gf[k][i])));
          d[i + 1] = __ffma2_rn(f2(kc), x[i + 1],
                                __ffma2_rn(f2(kd), w1, __fmul2_rn(f2(ka), gf[k][i + 1])));
          dw2[k][i] = __ffma2_rn(f2(kd), x[i], dw2[k][i]);
          dw2[k][i + 1] = __ffma2_rn(f2(kd), x[i + 1], dw2[k][i + 1]);
        }
        stg128(drow + (size_t)32 * k * VEC, pack2<T>(d));
      }
      release(slot, q);
    }
  }

  // ---- one dw partial row per CTA: the token streams' accumulators added in
  // stream order through shared memory (every issued row has been consumed,
  // so the ring is idle). CTA-uniform: if a wait ran out, every thread leaves.
  if (!__syncthreads_and(ok)) return;
  float* acc = reinterpret_cast<float*>(ring0);  // [streams][D] fp32
#pragma unroll
  for (int k = 0; k < CPL; ++k) {
    float* dst = acc + (size_t)gi * c.D + (size_t)(cb + 32 * k) * VEC;
#pragma unroll
    for (int i = 0; i < P; i += 2)
      *reinterpret_cast<float4*>(dst + 2 * i) =
          make_float4(dw2[k][i].x, dw2[k][i].y, dw2[k][i + 1].x, dw2[k][i + 1].y);
  }
  __syncthreads();
  float* prow = dw_partial + (size_t)blockIdx.x * c.D;
  for (int d = tid * 4; d < c.D; d += blockDim.x * 4) {
    float4 t = *reinterpret_cast<const float4*>(acc + d);
    for (int s = 1; s < streams; ++s) {
      const float4 u = *reinterpret_cast<const float4*>(acc + (size_t)s * c.D + d);
      t.x += u.x;
      t.y += u.y;
      t.z += u.z;
      t.w += u.w;
    }
    *reinterpret_cast<float4*>(prow + d) = t;
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

cudaError_t launch_stream_bwd(const StreamBwdCfg& c, int grid, int dtype, const void* v,
                              const void* w, int w_dtype, const void* g, const float* stats,
                              void* dv, float* dw_partial, cudaStream_t st);

}  // namespace sy
