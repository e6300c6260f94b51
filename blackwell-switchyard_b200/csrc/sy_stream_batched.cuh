// sy_stream_batched.cuh -- batched-query forward for shapes the register tile
// cannot hold (more than 16 sources, or rows too long for the tile at N > 9).
//
// out[s] = sum_n softmax_n(q_s . k_n) v_n for S <= 16 queries, k_n = v_n r_n,
// r_n = rsqrt(mean(v_n^2) + eps). K warps share a token, CPL 16-byte chunks
// per lane (K = D * itemsize / (512 CPL)), and the token's rows stream through the K warps'
// shared ring of row buffers (cp.async.bulk, one mbarrier each) twice:
//
//   pass A   v_0 .. v_{N-1} from HBM (evict-last hint): per row, the lane's
//            part of v_n . v_n and of q_s . v_n for every query (queries in
//            registers, loaded once per token from shared memory), one
//            reduce-scatter over the warp for every 32 / (S + 1) rows, the
//            warp's S + 1 sums per row to shared memory;
//   reduce   the K warps' sums added in warp order (named barrier), then one
//            warp per query: logits in lanes n < N, softmax, alpha_{s,n} to
//            shared memory;
//   pass B   v_0 .. v_{N-1} again (normally from L2, evict-first), per 8 / CPL
//            queries: out[s] += alpha_{s,n} v_n in fp32 registers, one 16-byte
//            store per query and chunk at the end (more queries: more sweeps).
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
  int row_chunks;  // 16-byte chunks per row: exactly 32 * cpl * kw
  int row_bytes;
  int kw;          // warps per token
  int cpl;         // chunks per lane (1, 2 or 4)
  int sb;          // query slots (4, 8 or 16; S <= sb, the rest are zero queries)
  int warps;       // per CTA, a multiple of kw
  int ring;        // row buffers per token stream
  float eps;
  float* mstats;   // optional (max logit, sum of exponentials) per (query, token)
  int raw;         // 1: unnormalised output sum_n exp(logit_n - max) v_n
};

constexpr int kStreamBatchedThreads = 512;
constexpr int kStreamBatchedMaxN = 32;  // lane n holds source n in the softmax
constexpr int kStreamBatchedMaxS = 16;
// pass B keeps 8 fp32 values per query and chunk: 8 / cpl queries per sweep
__host__ __device__ constexpr int stream_batched_qg(int cpl) { return 8 / cpl; }

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

// SB query slots, CPL chunks per lane. Pass A reduces RR = 32 / (SB + 1) rows
// per 32-wide reduce-scatter (3 at SB = 8).
template <typename T, int SB, int CPL>
__global__ void __launch_bounds__(kStreamBatchedThreads, 1)
    stream_batched_kernel(const T* __restrict__ v, const T* __restrict__ q, T* __restrict__ out,
                          const StreamBatchedCfg c) {
  constexpr int VEC = Dt<T>::kVec;
  constexpr int P = VEC / 2;
  constexpr int QG = stream_batched_qg(CPL);
  constexpr int W = SB + 1;   // values per row: v.v and SB dots
  constexpr int RR = 32 / W;  // rows per reduce-scatter
  static_assert(RR >= 1, "too many query slots");
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
      c.warps / K > 8 || c.ring < 2 || c.cpl != CPL || c.sb != SB ||
      c.row_chunks != 32 * CPL * K || RB != 16 * c.row_chunks || N < 1 ||
      N > kStreamBatchedMaxN || S < 1 || S > SB) {
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

  const int cb = wk * 32 * CPL + lane;  // this lane's chunks: cb + 32k
  const float inv_d = 1.f / (float)c.D;
  bool ok = true;
  int r = 0;
  int ring_slot = 0;        // slot and phase of stream row r (r mod R, (r / R) & 1)
  uint32_t ring_ph = 0;
  for (int j = 0; j < ntok && ok; ++j) {
    const long long tok = tok0 + tstride * j;
    // ---- pass A: v_n . v_n and q_s . v_n, this warp's part ----
    uint4 qr[SB][CPL];  // zero beyond S
#pragma unroll
    for (int s = 0; s < SB; ++s)
#pragma unroll
      for (int k = 0; k < CPL; ++k)
        qr[s][k] = s < S ? lds128(qsm + (size_t)s * RB + (cb + 32 * k) * 16)
                         : make_uint4(0u, 0u, 0u, 0u);
    for (int n0 = 0; n0 < N && ok; n0 += RR) {
      float a[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) a[i] = 0.f;
#pragma unroll
      for (int rr = 0; rr < RR; ++rr) {
        if (n0 + rr < N) {  // warp-uniform
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
          uint4 xu[CPL];
#pragma unroll
          for (int k = 0; k < CPL; ++k) xu[k] = lds128(ring + (size_t)slot * RB + (cb + 32 * k) * 16);
          release(slot, r);
          ++r;
          if constexpr (sizeof(T) == 2) {
            float2 acc = make_float2(0.f, 0.f);
#pragma unroll
            for (int k = 0; k < CPL; ++k) {
              mixfma2<T>(acc, xu[k].x, xu[k].x);
              mixfma2<T>(acc, xu[k].y, xu[k].y);
              mixfma2<T>(acc, xu[k].z, xu[k].z);
              mixfma2<T>(acc, xu[k].w, xu[k].w);
            }
            a[rr * W] = acc.x + acc.y;
#pragma unroll
            for (int s = 0; s < SB; ++s) {
              float2 d = make_float2(0.f, 0.f);
#pragma unroll
              for (int k = 0; k < CPL; ++k) {
                mixfma2<T>(d, qr[s][k].x, xu[k].x);
                mixfma2<T>(d, qr[s][k].y, xu[k].y);
                mixfma2<T>(d, qr[s][k].z, xu[k].z);
                mixfma2<T>(d, qr[s][k].w, xu[k].w);
              }
              a[rr * W + 1 + s] = d.x + d.y;
            }
          } else {
            float2 acc = make_float2(0.f, 0.f);
            float2 x[CPL][P];
#pragma unroll
            for (int k = 0; k < CPL; ++k) {
              unpack2<T>(xu[k], x[k]);
#pragma unroll
              for (int i = 0; i < P; ++i) acc = __ffma2_rn(x[k][i], x[k][i], acc);
            }
            a[rr * W] = acc.x + acc.y;
#pragma unroll
            for (int s = 0; s < SB; ++s) {
              float2 d = make_float2(0.f, 0.f);
#pragma unroll
              for (int k = 0; k < CPL; ++k) {
                float2 qf[P];
                unpack2<T>(qr[s][k], qf);
#pragma unroll
                for (int i = 0; i < P; ++i) d = __ffma2_rn(qf[i], x[k][i], d);
              }
              a[rr * W + 1 + s] = d.x + d.y;
            }
          }
        }
      }
      if (!ok) break;
      // lane L: the warp's sum of value L = (row n0 + L / W, value L mod W)
      const float tl = warp_reduce_scatter<32>(a, lane);
      const int rr = lane / W, i = lane - rr * W;
      if (rr < RR && n0 + rr < N && i < V) red[((size_t)(n0 + rr) * K + wk) * V + i] = tl;
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
      if (act) alpha[s * N + lane] = c.raw ? e : e / l;
      if (c.mstats != nullptr && lane == 0)
        reinterpret_cast<float2*>(c.mstats)[(size_t)s * c.BT + tok] = make_float2(m, l);
    }
    named_sync(1 + gi, 32 * K);

    // ---- pass B: QG queries per sweep over the rows ----
    for (int g0 = 0; g0 < S && ok; g0 += QG) {
      const int qn = S - g0 < QG ? S - g0 : QG;
      float2 o[QG][CPL][P];
#pragma unroll
      for (int qq = 0; qq < QG; ++qq)
#pragma unroll
        for (int k = 0; k < CPL; ++k)
#pragma unroll
          for (int i = 0; i < P; ++i) o[qq][k][i] = make_float2(0.f, 0.f);
      for (int n = 0; n < N; ++n, ++r) {
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
        float2 x[CPL][P];
#pragma unroll
        for (int k = 0; k < CPL; ++k)
          unpack2<T>(lds128(ring + (size_t)slot * RB + (cb + 32 * k) * 16), x[k]);
        release(slot, r);
        const float* ap = alpha + (size_t)g0 * N + n;
#pragma unroll
        for (int qq = 0; qq < QG; ++qq) {
          if (qq < qn) {
            const float al = ap[(size_t)qq * N];
#pragma unroll
            for (int k = 0; k < CPL; ++k)
#pragma unroll
              for (int i = 0; i < P; ++i) o[qq][k][i] = __ffma2_rn(f2(al), x[k][i], o[qq][k][i]);
          }
        }
      }
      if (!ok) break;
#pragma unroll
      for (int qq = 0; qq < QG; ++qq)
        if (qq < qn)
#pragma unroll
          for (int k = 0; k < CPL; ++k)
            stg128(out + ((size_t)(g0 + qq) * c.BT + tok) * c.D + (size_t)(cb + 32 * k) * VEC,
                   pack2<T>(o[qq][k]));
    }
  }
}

cudaError_t launch_stream_batched(const StreamBatchedCfg& c, int grid, int dtype, const void* v,
                                  const void* q, void* out, cudaStream_t st);

}  // namespace sy
