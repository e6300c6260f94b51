// sy_stream_batched.cuh -- batched-query forward for shapes the register tile
// cannot hold (more than 16 sources, or rows too long for the tile at N > 9).
//
// out[s] = sum_n softmax_n(q_s . k_n) v_n for S <= 16 queries, k_n = v_n r_n,
// r_n = rsqrt(mean(v_n^2) + eps). K = D * itemsize / 512 warps share a token,
// one 16-byte chunk per lane, and the token's rows stream through the K warps'
// shared ring of row buffers (cp.async.bulk, one mbarrier each) twice:
//
//   pass A   v_0 .. v_{N-1} from HBM (evict-last hint): per row, the lane's
//            part of v_n . v_n and of q_s . v_n for every query (queries in
//            registers, loaded once per token from shared memory), one
//            reduce-scatter over the warp, the warp's S + 1 sums to shared
//            memory;
//   reduce   the K warps' sums added in warp order (named barrier), then one
//            warp per query: logits in lanes n < N, softmax, alpha_{s,n} to
//            shared memory;
//   pass B   v_0 .. v_{N-1} again (normally from L2, evict-first), per 8
//            queries: out[s] += alpha_{s,n} v_n in fp32 registers, one 16-byte
//            store per query and lane at the end (S > 8: a second sweep).
//
// HBM traffic is the minimum, (N + S) rows per token; pass B's re-read stays
// on chip. Reference: the batched forward of src/switchyard/triton_op.py:
// 379-414 (resident) and its fallback loop :438-501 for the shapes handled
// here, with the math of reference.py:42-59 per query.
#pragma once

#include "sy_reg.cuh"

namespace sy {

struct StreamBatchedCfg {
  long long BT;
  int N, D, S;
  int row_chunks;  // 16-byte chunks per row: exactly 32 * kw
  int row_bytes;
  int kw;          // warps per token
  int warps;       // per CTA, a multiple of kw
  int ring;        // row buffers per token stream
  float eps;
};

constexpr int kStreamBatchedThreads = 512;
constexpr int kStreamBatchedMaxN = 32;  // lane n holds source n in the softmax
constexpr int kStreamBatchedMaxS = 16;
constexpr int kStreamBatchedQG = 8;     // queries per pass-B sweep (8 x 8 fp32 accumulators)

struct StreamBatchedSmem {
  size_t q_off, ring_off, bar_off, red_off, tot_off, alpha_off, cnt_off, total;
};

// queries (S rows), the streams' rings and barriers, the per-row warp sums
// [streams][N][kw][S+1], their totals [streams][N][S+1], alpha [streams][S][N]
// and the buffer-release counters [streams][ring].
__host__ __device__ inline StreamBatchedSmem stream_batched_smem_layout(const StreamBatchedCfg& c) {
  const int kw = c.kw > 0 ? c.kw : 1;
  const size_t streams = (size_t)(c.warps / kw);
  const size_t V = (size_t)c.S + 1;
  StreamBatchedSmem s;
  s.q_off = 0;
  s.ring_off = ((size_t)c.S * c.row_bytes + 127) / 128 * 128;
  s.bar_off = s.ring_off + streams * c.ring * c.row_bytes;
  s.red_off = s.bar_off + streams * c.ring * 8;
  s.tot_off = s.red_off + streams * c.N * kw * V * 4;
  s.alpha_off = s.tot_off + streams * c.N * V * 4;
  s.cnt_off = s.alpha_off + streams * c.S * c.N * 4;
  s.total = s.cnt_off + (streams * c.ring * 4 + 15) / 16 * 16;
  return s;
}

// M: the reduce-scatter width, 16 (S <= 15) or 32 (S = 16).
template <typename T, int M>
__global__ void __launch_bounds__(kStreamBatchedThreads, 1)
    stream_batched_kernel(const T* __restrict__ v, const T* __restrict__ q, T* __restrict__ out,
                          const StreamBatchedCfg c) {
  constexpr int VEC = Dt<T>::kVec;
  constexpr int P = VEC / 2;
  constexpr int QG = kStreamBatchedQG;
  constexpr int SMAX = kStreamBatchedMaxS;
  const StreamBatchedSmem L = stream_batched_smem_layout(c);
  unsigned char* qsm = sy_smem + L.q_off;
  unsigned char* ring0 = sy_smem + L.ring_off;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sy_smem + L.bar_off);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int wi = tid >> 5;
  const int K = c.kw, S = c.S, N = c.N, V = c.S + 1;
  const int RB = c.row_bytes;
  if (K < 2 || K > 16 || c.warps % K != 0 || c.warps != (int)(blockDim.x >> 5) ||
      c.warps / K > 8 || c.ring < 2 || c.row_chunks != 32 * K || RB != 16 * c.row_chunks ||
      N < 1 || N > kStreamBatchedMaxN || S < 2 || S > SMAX || V > M) {
    if (tid == 0) record_device_error(kDevErrBadPlan);
    return;
  }
  const int streams = c.warps / K;
  if (tid == 0) {
    for (int i = 0; i < streams * c.ring; ++i) mbar_init(&bars[i], 1);
    mbar_fence_init();
  }
  for (int i = tid; i < streams * c.ring; i += blockDim.x)
    reinterpret_cast<int*>(sy_smem + L.cnt_off)[i] = 0;
  {
    const uint4* src = reinterpret_cast<const uint4*>(q);
    uint4* dst = reinterpret_cast<uint4*>(qsm);
    for (int i = tid; i < S * c.row_chunks; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();

  const int gi = wi / K, wk = wi - gi * K;
  const long long tstride = (long long)gridDim.x * streams;
  const long long tok0 = blockIdx.x + (long long)gridDim.x * gi;
  const int ntok = tok0 < c.BT ? (int)((c.BT - 1 - tok0) / tstride) + 1 : 0;
  const int ngrp = (S + QG - 1) / QG;
  const int LT = N * (1 + ngrp);  // stream rows per token
  const int nrows = ntok * LT;    // the planner keeps this below 2^31
  unsigned char* ring = ring0 + (size_t)gi * c.ring * RB;
  uint64_t* bar = bars + gi * c.ring;
  int* cnt = reinterpret_cast<int*>(sy_smem + L.cnt_off) + gi * c.ring;
  float* red = reinterpret_cast<float*>(sy_smem + L.red_off) + (size_t)gi * N * K * V;
  float* tot = reinterpret_cast<float*>(sy_smem + L.tot_off) + (size_t)gi * N * V;
  float* alpha = reinterpret_cast<float*>(sy_smem + L.alpha_off) + (size_t)gi * S * N;
  const size_t nstride = (size_t)c.BT * RB;
  const unsigned char* vb = reinterpret_cast<const unsigned char*>(v);

  // stream row r: row (r mod LT) mod N of token r / LT; its first N rows per
  // token are pass A (kept in L2 for the sweeps that follow)
  auto issue_row = [&](int slot_, int r) {
    if (r >= nrows) return;
    const int jj = r / LT, ii = r - jj * LT;
    const int nn = ii % N;
    const unsigned char* src = vb + (size_t)nn * nstride + (size_t)(tok0 + tstride * jj) * RB;
    mbar_arrive_expect_tx(&bar[slot_], (uint32_t)RB);
    bulk_g2s(ring + (size_t)slot_ * RB, src, (uint32_t)RB, &bar[slot_],
             ii < N ? policy_evict_last() : policy_evict_first());
  };
  auto release = [&](int slot_, int r) {
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      if (atomicAdd(&cnt[slot_], 1) == K - 1) {
        cnt[slot_] = 0;
        __threadfence_block();
        fence_proxy_async();
        issue_row(slot_, r + c.ring);
      }
    }
  };
  if (wk == 0 && lane == 0)
    for (int s = 0; s < c.ring; ++s) issue_row(s, s);

  const int ch = wk * 32 + lane;  // this lane's chunk of every row
  const float inv_d = 1.f / (float)c.D;
  bool ok = true;
  int r = 0;
  for (int j = 0; j < ntok && ok; ++j) {
    const long long tok = tok0 + tstride * j;
    // ---- pass A: v_n . v_n and q_s . v_n, this warp's part ----
    uint4 qr[SMAX];
#pragma unroll
    for (int s = 0; s < SMAX; ++s)
      qr[s] = s < S ? lds128(qsm + (size_t)s * RB + ch * 16) : make_uint4(0u, 0u, 0u, 0u);
    for (int n = 0; n < N; ++n, ++r) {
      const int slot = r % c.ring;
      if (!mbar_wait(&bar[slot], (uint32_t)((r / c.ring) & 1))) {
        ok = false;
        break;
      }
      const uint4 xu = lds128(ring + (size_t)slot * RB + ch * 16);
      release(slot, r);
      float a[M];
#pragma unroll
      for (int i = 0; i < M; ++i) a[i] = 0.f;
      if constexpr (sizeof(T) == 2) {
        float2 acc = make_float2(0.f, 0.f);
        mixfma2<T>(acc, xu.x, xu.x);
        mixfma2<T>(acc, xu.y, xu.y);
        mixfma2<T>(acc, xu.z, xu.z);
        mixfma2<T>(acc, xu.w, xu.w);
        a[0] = acc.x + acc.y;
#pragma unroll
        for (int s = 0; s < SMAX && s + 1 < M; ++s) {
          if (s < S) {
            float2 d = make_float2(0.f, 0.f);
            mixfma2<T>(d, qr[s].x, xu.x);
            mixfma2<T>(d, qr[s].y, xu.y);
            mixfma2<T>(d, qr[s].z, xu.z);
            mixfma2<T>(d, qr[s].w, xu.w);
            a[1 + s] = d.x + d.y;
          }
        }
      } else {
        float2 x[P];
        unpack2<T>(xu, x);
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < P; ++i) acc = __ffma2_rn(x[i], x[i], acc);
        a[0] = acc.x + acc.y;
#pragma unroll
        for (int s = 0; s < SMAX && s + 1 < M; ++s) {
          if (s < S) {
            float2 qf[P];
            unpack2<T>(qr[s], qf);
            float2 d = make_float2(0.f, 0.f);
#pragma unroll
            for (int i = 0; i < P; ++i) d = __ffma2_rn(qf[i], x[i], d);
            a[1 + s] = d.x + d.y;
          }
        }
      }
      const float tl = warp_reduce_scatter<M>(a, lane);
      const int vi = rs_index<M>(lane);
      if (vi < V && (M == 32 || (lane & 1) == 0)) red[((size_t)n * K + wk) * V + vi] = tl;
    }
    if (!ok) break;
    named_sync(1 + gi, 32 * K);

    // ---- totals over the K warps, in warp order ----
    for (int idx = wk * 32 + lane; idx < N * V; idx += 32 * K) {
      const int n = idx / V, i = idx - n * V;
      const float* rp = red + (size_t)n * K * V + i;
      float t = rp[0];
      for (int k = 1; k < K; ++k) t += rp[(size_t)k * V];
      tot[idx] = t;
    }
    named_sync(1 + gi, 32 * K);

    // ---- softmax: warp wk takes queries wk, wk + K, ...; lane n source n ----
    for (int s = wk; s < S; s += K) {
      const bool act = lane < N;
      float logit = -INFINITY;
      if (act) {
        const float rn = rsqrtf(tot[lane * V] * inv_d + c.eps);
        logit = tot[lane * V + 1 + s] * rn;
      }
      const float m = warp_max(logit);
      const float e = act ? expf(logit - m) : 0.f;
      const float l = warp_sum(e);
      if (act) alpha[s * N + lane] = e / l;
    }
    named_sync(1 + gi, 32 * K);

    // ---- pass B: up to QG queries per sweep over the rows ----
    for (int g0 = 0; g0 < S && ok; g0 += QG) {
      const int qn = S - g0 < QG ? S - g0 : QG;
      float2 o[QG][P];
#pragma unroll
      for (int qq = 0; qq < QG; ++qq)
#pragma unroll
        for (int i = 0; i < P; ++i) o[qq][i] = make_float2(0.f, 0.f);
      for (int n = 0; n < N; ++n, ++r) {
        const int slot = r % c.ring;
        if (!mbar_wait(&bar[slot], (uint32_t)((r / c.ring) & 1))) {
          ok = false;
          break;
        }
        float2 x[P];
        unpack2<T>(lds128(ring + (size_t)slot * RB + ch * 16), x);
        release(slot, r);
        const float* ap = alpha + (size_t)g0 * N + n;
#pragma unroll
        for (int qq = 0; qq < QG; ++qq) {
          if (qq < qn) {
            const float al = ap[(size_t)qq * N];
#pragma unroll
            for (int i = 0; i < P; ++i) o[qq][i] = __ffma2_rn(f2(al), x[i], o[qq][i]);
          }
        }
      }
      if (!ok) break;
#pragma unroll
      for (int qq = 0; qq < QG; ++qq)
        if (qq < qn)
          stg128(out + ((size_t)(g0 + qq) * c.BT + tok) * c.D + (size_t)ch * VEC, pack2<T>(o[qq]));
    }
  }
}

cudaError_t launch_stream_batched(const StreamBatchedCfg& c, int grid, int dtype, const void* v,
                                  const void* q, void* out, cudaStream_t st);

}  // namespace sy
