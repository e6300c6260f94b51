// sy_stream.cuh -- "row stream" forward: one warp per token, online softmax.
//
// Every warp of the persistent CTA works alone: it takes tokens
// k = cta + grid * (warp + W * j), j = 0, 1, ... (so each SM gets an equal
// share and, within it, its W warps take turns), and streams the token's N
// source rows one at a time through its own ring of R shared-memory row
// buffers, filled by cp.async.bulk (one mbarrier per buffer). Per row the
// lane's CPL 16-byte chunks go to registers as fp32 (the buffer is refilled
// with the row R ahead right away), then
//
//   dot = w.v_n, ssq = v_n.v_n         packed fp32 FMA, butterfly over the warp
//   logit = dot * rsqrt(ssq/D + eps)    (no 1/sqrt(D); bitwise equal in all lanes)
//   online softmax over n:             if logit > m: o = o*exp(m-logit) + v_n,
//                                      l = l*exp(m-logit) + 1, m = logit
//                                      else: p = exp(logit-m), o += p*v_n, l += p
//
// and after the last row out = o / l, rounded once. There is no block-level
// barrier anywhere, the source count is a run-time loop (any N), and the
// statistics (logit_n, r_n, m, lse = m + log l) fall out of the same pass.
// w is converted to fp32 once per CTA into shared memory, stored as VEC/4
// planes of float4 per chunk so the per-row reads are conflict-free.
//
// Reference math: src/switchyard/reference.py:42-59; the two-phase merge of
// partial softmaxes it follows is reference.py:219-233 applied one row at a time.
#pragma once

#include "sy_launch.cuh"
#include "sy_tile.cuh"

namespace sy {

extern __shared__ __align__(1024) unsigned char sy_smem[];

struct StreamCfg {
  long long BT;
  int N, D;
  int row_chunks;    // 16-byte chunks per row
  int row_bytes;     // padded to a multiple of 16 (rows are contiguous in HBM)
  int warps;         // W per CTA
  int ring;          // R row buffers per token stream (per warp, or per warp group)
  int stats_stride;
  int reread;        // 1: second pass reads the row again from shared memory
  int kw;            // warps sharing one token (re-read variant; 0 or 1: one)
  float eps;
};

struct StreamSmem {
  size_t w_off, ring_off, bar_off, xch_off, cnt_off, zero_off, total;
};

// fp32 w, then the rings of the W / kw token streams, their full barriers, and
// (kw > 1) the per-row exchange of partial sums and the buffer-release counters.
__host__ __device__ inline StreamSmem stream_smem_layout(const StreamCfg& c) {
  const int kw = c.kw > 1 ? c.kw : 1;
  const size_t streams = (size_t)(c.warps / kw);
  StreamSmem s;
  s.w_off = 0;                                                   // fp32 w[D]
  s.ring_off = ((size_t)c.D * 4 + 127) / 128 * 128;              // streams * R rows
  s.bar_off = s.ring_off + streams * c.ring * c.row_bytes;
  // the full barriers plus w's, rounded up to 16 bytes (the zero pad below is
  // read and written as one 16-byte vector)
  s.xch_off = s.bar_off + ((streams * c.ring + 1) * 8 + 15) / 16 * 16;  // float2 [streams][2][kw]
  s.cnt_off = s.xch_off + (kw > 1 ? streams * 2 * kw * 8 : 0);   // int [streams][R]
  s.zero_off = s.cnt_off + (kw > 1 ? (streams * c.ring * 4 + 15) / 16 * 16 : 0);
  s.total = s.zero_off + 16;
  return s;
}

#ifndef SY_TUNE_STREAM8_THREADS
#define SY_TUNE_STREAM8_THREADS 384
#endif

// Threads per CTA for CPL chunks per lane. The fp32 row and the fp32 output
// accumulator take 2 * 4 * CPL registers per lane (64 each at CPL=8 bf16),
// so CPL <= 4 runs 16 warps per SM and CPL = 8 twelve (168 registers each).
// REREAD drops the fp32 row from the registers (the second pass reads it from
// shared memory again), which leaves room for 14 warps at CPL = 8.
#ifndef SY_TUNE_REREAD_WARPS
#define SY_TUNE_REREAD_WARPS 14
#endif
// Up to 14 warps. (The register file is split between the SM's four warp
// schedulers, so anything over 12 warps caps a thread at 128 registers.)
constexpr int kStreamRereadThreads = 32 * SY_TUNE_REREAD_WARPS;
__host__ __device__ constexpr int stream_threads(int cpl, bool reread = false) {
  return reread ? kStreamRereadThreads : (cpl <= 4 ? 512 : SY_TUNE_STREAM8_THREADS);
}

// FULL: the row is exactly 32 * CPL chunks (D = 256, 512, 1024, 2048 bf16),
// so no lane needs a validity predicate.

template <typename T, int CPL, bool SOL, bool FULL>
__global__ void __launch_bounds__(stream_threads(CPL), 1)
    stream_fwd_kernel(const T* __restrict__ v, const void* __restrict__ w, int w_dtype,
                      T* __restrict__ out, float* __restrict__ stats, const StreamCfg c) {
  constexpr int VEC = Dt<T>::kVec;
  constexpr int P = VEC / 2;
  const StreamSmem L = stream_smem_layout(c);
  float* wsm = reinterpret_cast<float*>(sy_smem + L.w_off);
  unsigned char* ring0 = sy_smem + L.ring_off;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sy_smem + L.bar_off);
  const unsigned char* zero_pad = sy_smem + L.zero_off;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int wi = tid >> 5;
  if (c.warps != (int)(blockDim.x >> 5) || c.ring < 1) {
    if (tid == 0) record_device_error(kDevErrBadPlan);
    return;
  }

  if (tid == 0) {
    for (int i = 0; i < c.warps * c.ring; ++i) mbar_init(&bars[i], 1);
    *reinterpret_cast<uint4*>(sy_smem + L.zero_off) = make_uint4(0u, 0u, 0u, 0u);
    mbar_fence_init();
  }
  // plane p of chunk ch holds w[ch*VEC + 4p .. 4p+3] at wsm[(p*chunks + ch)*4]
  if constexpr (!SOL)
    for (int d = tid; d < c.D; d += blockDim.x) {
      const int ch = d / VEC, e = d - ch * VEC;
      wsm[((e >> 2) * c.row_chunks + ch) * 4 + (e & 3)] = load_any(w, w_dtype, d);
    }
  __syncthreads();

  const long long grid = gridDim.x;
  const long long tok0 = blockIdx.x + grid * wi;
  const long long tstride = grid * c.warps;
  const long long ntok = tok0 < c.BT ? (c.BT - 1 - tok0) / tstride + 1 : 0;
  const long long nrows = ntok * c.N;  // this warp's row stream
  unsigned char* ring = ring0 + (size_t)wi * c.ring * c.row_bytes;
  uint64_t* bar = bars + wi * c.ring;
  const uint64_t pol = policy_evict_first();
  const size_t nstride = (size_t)c.BT * c.row_bytes;
  const unsigned char* vb = reinterpret_cast<const unsigned char*>(v);

  // The row stream is token-major: row q is source (q mod N) of the warp's
  // token q / N. (iss_j, iss_n) is the next row to issue into the ring.
  long long iss_j = 0;
  int iss_n = 0;
  long long issued = 0;
  auto issue_next = [&](int slot_) {
    if (lane == 0) {
      const long long tok = tok0 + tstride * iss_j;
      mbar_arrive_expect_tx(&bar[slot_], (uint32_t)c.row_bytes);
      bulk_g2s(ring + (size_t)slot_ * c.row_bytes,
               vb + (size_t)iss_n * nstride + (size_t)tok * c.row_bytes, (uint32_t)c.row_bytes,
               &bar[slot_], pol);
    }
    ++issued;
    if (++iss_n == c.N) {
      iss_n = 0;
      ++iss_j;
    }
  };
  for (int s = 0; s < c.ring && issued < nrows; ++s) issue_next(s);
  pdl_trigger();

  // Lane-chunk k of a row is chunk lane + 32k; past the row end (only when
  // !FULL) it reads the zero pad instead.
  auto cval = [&](int k) { return FULL || lane + 32 * k < c.row_chunks; };
  const float inv_d = 1.f / (float)c.D;

  int slot = 0;
  uint32_t ph = 0;
  for (long long j = 0; j < ntok; ++j) {
    const long long tok = tok0 + tstride * j;
    float* st = stats != nullptr ? stats + tok * c.stats_stride : nullptr;
    float2 o[CPL][P];
    float m = 0.f, l = 0.f;
    for (int n = 0; n < c.N; ++n) {
      if (!mbar_wait(&bar[slot], ph)) return;
      const unsigned char* row = ring + (size_t)slot * c.row_bytes;
      float2 x[CPL][P];
#pragma unroll
      for (int k = 0; k < CPL; ++k)
        unpack2<T>(lds128(cval(k) ? row + (lane + 32 * k) * 16 : zero_pad), x[k]);
      __syncwarp();
      if (issued < nrows) {
        if (lane == 0) fence_proxy_async();
        issue_next(slot);
      }
      if (++slot == c.ring) {
        slot = 0;
        ph ^= 1u;
      }

      if constexpr (SOL) {
#pragma unroll
        for (int k = 0; k < CPL; ++k)
#pragma unroll
          for (int i = 0; i < P; ++i) o[k][i] = n == 0 ? x[k][i] : __fadd2_rn(o[k][i], x[k][i]);
        continue;
      } else {
        // dot and sum of squares: two independent accumulator pairs each
        float2 dacc[2], sacc[2];
#pragma unroll
        for (int a = 0; a < 2; ++a) dacc[a] = sacc[a] = make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < CPL; ++k) {
          const float4* wp = reinterpret_cast<const float4*>(wsm) + (lane + 32 * k);
#pragma unroll
          for (int i = 0; i < P; i += 2) {
            const float4 wv =
                cval(k) ? wp[(i / 2) * c.row_chunks] : make_float4(0.f, 0.f, 0.f, 0.f);
            dacc[0] = __ffma2_rn(make_float2(wv.x, wv.y), x[k][i], dacc[0]);
            sacc[0] = __ffma2_rn(x[k][i], x[k][i], sacc[0]);
            dacc[1] = __ffma2_rn(make_float2(wv.z, wv.w), x[k][i + 1], dacc[1]);
            sacc[1] = __ffma2_rn(x[k][i + 1], x[k][i + 1], sacc[1]);
          }
        }
        const float2 d2 = __fadd2_rn(dacc[0], dacc[1]);
        const float2 s2 = __fadd2_rn(sacc[0], sacc[1]);
        float dot = d2.x + d2.y, ssq = s2.x + s2.y;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
          dot += __shfl_xor_sync(kFull, dot, off);
          ssq += __shfl_xor_sync(kFull, ssq, off);
        }
        const float r = rsqrtf(ssq * inv_d + c.eps);
        const float logit = dot * r;
        if (st != nullptr && lane == 0) {
          st[n] = logit;
          st[c.N + n] = r;
        }
        if (n == 0) {
          m = logit;
          l = 1.f;
#pragma unroll
          for (int k = 0; k < CPL; ++k)
#pragma unroll
            for (int i = 0; i < P; ++i) o[k][i] = x[k][i];
        } else if (logit > m) {  // warp-uniform: logit is bitwise equal in all lanes
          const float sc = expf(m - logit);
          m = logit;
          l = fmaf(l, sc, 1.f);
#pragma unroll
          for (int k = 0; k < CPL; ++k)
#pragma unroll
            for (int i = 0; i < P; ++i) o[k][i] = __ffma2_rn(o[k][i], f2(sc), x[k][i]);
        } else {
          const float p = expf(logit - m);
          l += p;
#pragma unroll
          for (int k = 0; k < CPL; ++k)
#pragma unroll
            for (int i = 0; i < P; ++i) o[k][i] = __ffma2_rn(f2(p), x[k][i], o[k][i]);
        }
      }
    }
    if constexpr (!SOL) {
      if (st != nullptr && lane == 0) {
        st[2 * c.N] = m;
        st[2 * c.N + 1] = m + logf(l);
      }
      const float inv = 1.f / l;
#pragma unroll
      for (int k = 0; k < CPL; ++k)
#pragma unroll
        for (int i = 0; i < P; ++i) o[k][i] = __fmul2_rn(o[k][i], f2(inv));
    }
    T* orow = out + tok * c.D;
#pragma unroll
    for (int k = 0; k < CPL; ++k)
      if (cval(k)) stg128(orow + (lane + 32 * k) * VEC, pack2<T>(o[k]));
  }
}

// Stage w in shared memory for the re-read kernels. MIX: in its own 16-bit
// type, row layout (chunk ch at byte 16 ch), copied in 16-byte chunks when w is
// aligned; otherwise fp32 in VEC/4 planes of float4 per chunk (plane p of
// chunk ch at float4 p * rc + ch), conflict-free for lane-consecutive chunks.
template <typename T, bool MIX>
__device__ __forceinline__ void stage_w(float* wsm, const void* w, int w_dtype, int D, int rc) {
  constexpr int VEC = Dt<T>::kVec;
  if constexpr (MIX) {
    if ((reinterpret_cast<uintptr_t>(w) & 15u) == 0) {
      for (int ch = threadIdx.x; ch < rc; ch += blockDim.x)
        reinterpret_cast<uint4*>(wsm)[ch] = reinterpret_cast<const uint4*>(w)[ch];
    } else {
      for (int d = threadIdx.x; d < D; d += blockDim.x)
        reinterpret_cast<T*>(wsm)[d] = reinterpret_cast<const T*>(w)[d];
    }
  } else {
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      const int ch = d / VEC, e = d - ch * VEC;
      wsm[((e >> 2) * rc + ch) * 4 + (e & 3)] = load_any(w, w_dtype, d);
    }
  }
}

// Re-read variant of the row stream (8 chunks per lane: 4 KiB rows, or 4: 2 KiB
// rows). Per row,
// pass 1 reads the lane's chunks from the row buffer for the dot and the sum
// of squares only; after the online-softmax update pass 2 reads them again
// for o (o += p * v_n; a new maximum first rescales o and enters v_n with
// p = 1), and only then is the buffer refilled. The
// fp32 row never lives in registers and the bookkeeping is kept to 32-bit
// counters and one running source pointer, so 14 warps (128 registers) fit
// on an SM: with whole tokens per warp that balances 28 tokens per SM as
// 2 per warp (the representative 4096 tokens on 148 SMs).
template <typename T, int CPL, bool FULL, bool MIX>
__global__ void __launch_bounds__(kStreamRereadThreads, 1)
    stream_fwd_reread_kernel(const T* __restrict__ v, const void* __restrict__ w, int w_dtype,
                             T* __restrict__ out, float* __restrict__ stats, const StreamCfg c) {
  static_assert(CPL == 4 || CPL == 8, "4 or 8 chunks per lane");
  constexpr int VEC = Dt<T>::kVec;
  constexpr int P = VEC / 2;
  const int RC = FULL ? 32 * CPL : c.row_chunks;  // chunks per row
  const int RB = FULL ? 16 * 32 * CPL : c.row_bytes;
  const StreamSmem L = stream_smem_layout(c);
  float* wsm = reinterpret_cast<float*>(sy_smem + L.w_off);
  unsigned char* ring0 = sy_smem + L.ring_off;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sy_smem + L.bar_off);
  const unsigned char* zero_pad = sy_smem + L.zero_off;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int wi = tid >> 5;
  if (c.warps != (int)(blockDim.x >> 5) || c.ring < 1 || !c.reread) {
    if (tid == 0) record_device_error(kDevErrBadPlan);
    return;
  }
  // A 16-bit w in the sources' type (MIX) is already in the row layout: one
  // bulk copy, the first in the queue, so the rings start filling at once.
  // Otherwise w is staged by the threads before the rings start filling
  // (issued after the bulk copies, its loads would wait behind them).
  uint64_t* wbar = bars + c.warps * c.ring;
  const bool wtma = MIX && (reinterpret_cast<uintptr_t>(w) & 15u) == 0;
  if (tid == 0) {
    for (int i = 0; i < c.warps * c.ring + 1; ++i) mbar_init(&bars[i], 1);
    *reinterpret_cast<uint4*>(sy_smem + L.zero_off) = make_uint4(0u, 0u, 0u, 0u);
    mbar_fence_init();
    if (wtma) {
      mbar_arrive_expect_tx(wbar, (uint32_t)c.row_bytes);
      bulk_g2s(wsm, w, (uint32_t)c.row_bytes, wbar, policy_evict_last());
    }
  }
  if (!wtma) stage_w<T, MIX>(wsm, w, w_dtype, c.D, c.row_chunks);
  __syncthreads();

  // This warp's tokens: tok0 + tstride * j, j < ntok (fewer than 2^31 rows
  // per warp: the planner checks it).
  const long long tstride = (long long)gridDim.x * c.warps;
  const long long tok0 = blockIdx.x + (long long)gridDim.x * wi;
  const int ntok = tok0 < c.BT ? (int)((c.BT - 1 - tok0) / tstride) + 1 : 0;
  unsigned char* ring = ring0 + (size_t)wi * c.ring * RB;
  uint64_t* bar = bars + wi * c.ring;
  // next row to issue: source iss_n of the warp's token iss_j, at src
  int iss_j = 0, iss_n = 0;
  const unsigned char* src = reinterpret_cast<const unsigned char*>(v) + (size_t)tok0 * RB;
  auto issue_next = [&](int slot_) {
    if (iss_j >= ntok) return;
    const size_t nstride = (size_t)c.BT * RB;
    if (lane == 0) {
      mbar_arrive_expect_tx(&bar[slot_], (uint32_t)RB);
      bulk_g2s(ring + (size_t)slot_ * RB, src, (uint32_t)RB, &bar[slot_], policy_evict_first());
    }
    if (++iss_n == c.N) {
      iss_n = 0;
      ++iss_j;
      src += (size_t)gridDim.x * c.warps * RB - (size_t)(c.N - 1) * nstride;
    } else {
      src += nstride;
    }
  };
  for (int s = 0; s < c.ring; ++s) issue_next(s);
  pdl_trigger();  // every CTA is resident: the next kernel may queue for the SMs
  if (wtma && !mbar_wait(wbar, 0u)) return;

  auto cval = [&](int k) { return FULL || lane + 32 * k < RC; };
  const float inv_d = 1.f / (float)c.D;
  int slot = 0;
  uint32_t ph = 0;
  for (int j = 0; j < ntok; ++j) {
    float2 o[CPL][P];
#pragma unroll
    for (int k = 0; k < CPL; ++k)
#pragma unroll
      for (int i = 0; i < P; ++i) o[k][i] = make_float2(0.f, 0.f);
    // mref: the reference the weights are taken against (o and l hold
    // sum exp(logit - mref) v and sum exp(logit - mref)); mx: the max logit.
    float mref = 0.f, mx = 0.f, l = 0.f;
    float lane_logit = 0.f, lane_r = 0.f;  // row `lane`'s statistics (lane < N)
    float* st = stats != nullptr ? stats + (tok0 + tstride * j) * c.stats_stride : nullptr;
    for (int n = 0; n < c.N; ++n) {
      if (!mbar_wait(&bar[slot], ph)) return;
      const unsigned char* row = ring + (size_t)slot * RB;
      // pass 1: dot and sum of squares, two independent accumulator pairs each
      constexpr int A = P < 2 ? P : 2;
      float2 dacc[A], sacc[A];
#pragma unroll
      for (int i = 0; i < A; ++i) dacc[i] = sacc[i] = make_float2(0.f, 0.f);
#pragma unroll
      for (int k = 0; k < CPL; ++k) {
        if (k % 4 == 0 && k > 0) __syncwarp();  // bounds the loads hoisted ahead (registers)
        if constexpr (MIX) {
          // the same products and accumulation order as below, on the packed
          // 16-bit halves (pair i of the chunk is word i)
          const uint4 xu = lds128(cval(k) ? row + (lane + 32 * k) * 16 : zero_pad);
          const uint4 wu = lds128(cval(k) ? reinterpret_cast<const unsigned char*>(wsm) +
                                                (lane + 32 * k) * 16
                                          : zero_pad);
          mixfma2<T>(dacc[0], wu.x, xu.x);
          mixfma2<T>(sacc[0], xu.x, xu.x);
          mixfma2<T>(dacc[A - 1], wu.y, xu.y);
          mixfma2<T>(sacc[A - 1], xu.y, xu.y);
          mixfma2<T>(dacc[0], wu.z, xu.z);
          mixfma2<T>(sacc[0], xu.z, xu.z);
          mixfma2<T>(dacc[A - 1], wu.w, xu.w);
          mixfma2<T>(sacc[A - 1], xu.w, xu.w);
        } else {
          float2 x[P];
          unpack2<T>(lds128(cval(k) ? row + (lane + 32 * k) * 16 : zero_pad), x);
          const float4* wp = reinterpret_cast<const float4*>(wsm) + (lane + 32 * k);
#pragma unroll
          for (int i = 0; i < P; i += 2) {
            const float4 wv = cval(k) ? wp[(i / 2) * RC] : make_float4(0.f, 0.f, 0.f, 0.f);
            dacc[0] = __ffma2_rn(make_float2(wv.x, wv.y), x[i], dacc[0]);
            sacc[0] = __ffma2_rn(x[i], x[i], sacc[0]);
            dacc[A - 1] = __ffma2_rn(make_float2(wv.z, wv.w), x[i + 1], dacc[A - 1]);
            sacc[A - 1] = __ffma2_rn(x[i + 1], x[i + 1], sacc[A - 1]);
          }
        }
      }
#pragma unroll
      for (int i = 1; i < A; ++i) {
        dacc[0] = __fadd2_rn(dacc[0], dacc[i]);
        sacc[0] = __fadd2_rn(sacc[0], sacc[i]);
      }
      // (dot, ssq) as one pair through the butterfly
      float2 ds = make_float2(dacc[0].x + dacc[0].y, sacc[0].x + sacc[0].y);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
        ds = __fadd2_rn(ds, make_float2(__shfl_xor_sync(kFull, ds.x, off),
                                        __shfl_xor_sync(kFull, ds.y, off)));
      const float r = rsqrtf(ds.y * inv_d + c.eps);
      const float logit = ds.x * r;
      if (lane == n) {  // (never for n >= 32: those rows are written directly below)
        lane_logit = logit;
        lane_r = r;
      }
      if (n >= 32 && st != nullptr && lane == 0) {  // rows past 32: written directly
        st[n] = logit;
        st[c.N + n] = r;
      }
      // Online softmax, warp-uniform (logit is bitwise equal in all lanes).
      // Weights are exp(logit - mref); mref only moves when a logit exceeds it
      // by more than kRescaleGap, so o is rescaled rarely and the weights stay
      // below e^kRescaleGap (no overflow in fp32).
      constexpr float kRescaleGap = 8.f;
      float wgt = 1.f;
      if (n == 0) {
        mref = mx = logit;
        l = 1.f;
      } else {
        mx = fmaxf(mx, logit);
        if (logit > mref + kRescaleGap) {
          const float sc = expf(mref - logit);
          mref = logit;
          l = fmaf(l, sc, 1.f);
#pragma unroll
          for (int k = 0; k < CPL; ++k)
#pragma unroll
            for (int i = 0; i < P; ++i) o[k][i] = __fmul2_rn(o[k][i], f2(sc));
        } else {
          wgt = expf(logit - mref);
          l += wgt;
        }
      }
      // pass 2: the row again, into o (o is 0 before the first row)
#pragma unroll
      for (int k = 0; k < CPL; ++k) {
        if (k % 4 == 0 && k > 0) __syncwarp();
        float2 x[P];
        unpack2<T>(lds128(cval(k) ? row + (lane + 32 * k) * 16 : zero_pad), x);
#pragma unroll
        for (int i = 0; i < P; ++i) o[k][i] = __ffma2_rn(f2(wgt), x[i], o[k][i]);
      }
      __syncwarp();
      if (lane == 0) fence_proxy_async();
      issue_next(slot);
      if (++slot == c.ring) {
        slot = 0;
        ph ^= 1u;
      }
    }
    if (st != nullptr) {
      if (lane < c.N) {
        st[lane] = lane_logit;
        st[c.N + lane] = lane_r;
      }
      if (lane == 0) {
        st[2 * c.N] = mx;
        st[2 * c.N + 1] = mref + logf(l);
      }
    }
    const float inv = 1.f / l;
    T* orow = out + (tok0 + tstride * j) * c.D;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
#pragma unroll
      for (int i = 0; i < P; ++i) o[k][i] = __fmul2_rn(o[k][i], f2(inv));
      if (cval(k)) stg128(orow + (lane + 32 * k) * VEC, pack2<T>(o[k]));
    }
  }
}

// Split variant of the re-read row stream for rows of K * 4 KiB (K = 2, 4, 8: D =
// 4096 / 8192 / 16384 bf16): K warps share each token, warp k taking chunks
// 256k .. 256k+255 of every row (8 per lane). Per row each warp reduces its
// part of (dot, ssq) over its lanes; lane 0 publishes the pair, the K warps
// meet at a named barrier and every warp adds the K pairs in warp order, so all
// of them hold the bitwise-same logit, softmax state and weight. The row buffer
// is shared: each warp, after its second pass over its part, adds one to the
// buffer's counter and the warp that completes the count refills it (with the
// group's row a ring-length ahead) -- no second barrier per row.
template <typename T, int K, bool MIX>
__global__ void __launch_bounds__(kStreamRereadThreads, 1)
    stream_fwd_split_kernel(const T* __restrict__ v, const void* __restrict__ w, int w_dtype,
                            T* __restrict__ out, float* __restrict__ stats, const StreamCfg c) {
  constexpr int CPL = 8;
  constexpr int VEC = Dt<T>::kVec;
  constexpr int P = VEC / 2;
  constexpr int RC = 256 * K;  // chunks per row
  constexpr int RB = 16 * RC;  // bytes per row
  const StreamSmem L = stream_smem_layout(c);
  float* wsm = reinterpret_cast<float*>(sy_smem + L.w_off);
  unsigned char* ring0 = sy_smem + L.ring_off;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sy_smem + L.bar_off);
  float2* xch0 = reinterpret_cast<float2*>(sy_smem + L.xch_off);
  int* cnt0 = reinterpret_cast<int*>(sy_smem + L.cnt_off);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int wi = tid >> 5;
  const int streams = c.warps / K;
  if (c.kw != K || c.warps % K != 0 || c.warps != (int)(blockDim.x >> 5) || c.ring < 1 ||
      !c.reread || c.row_chunks != RC || c.row_bytes != RB) {
    if (tid == 0) record_device_error(kDevErrBadPlan);
    return;
  }
  uint64_t* wbar = bars + streams * c.ring;  // w as one bulk copy (see the re-read kernel)
  const bool wtma = MIX && (reinterpret_cast<uintptr_t>(w) & 15u) == 0;
  if (tid == 0) {
    for (int i = 0; i < streams * c.ring + 1; ++i) mbar_init(&bars[i], 1);
    mbar_fence_init();
    if (wtma) {
      mbar_arrive_expect_tx(wbar, (uint32_t)RB);
      bulk_g2s(wsm, w, (uint32_t)RB, wbar, policy_evict_last());
    }
  }
  for (int i = tid; i < streams * c.ring; i += blockDim.x) cnt0[i] = 0;
  if (!wtma) stage_w<T, MIX>(wsm, w, w_dtype, c.D, RC);
  __syncthreads();

  const int gi = wi / K, wk = wi - gi * K;
  const long long tstride = (long long)gridDim.x * streams;
  const long long tok0 = blockIdx.x + (long long)gridDim.x * gi;
  const int ntok = tok0 < c.BT ? (int)((c.BT - 1 - tok0) / tstride) + 1 : 0;
  const int nrows = ntok * c.N;  // the planner keeps this below 2^31
  unsigned char* ring = ring0 + (size_t)gi * c.ring * RB;
  uint64_t* bar = bars + gi * c.ring;
  float2* xch = xch0 + gi * 2 * K;
  int* cnt = cnt0 + gi * c.ring;
  const size_t nstride = (size_t)c.BT * RB;
  // row q of this stream: source q mod N of token q / N
  auto issue_row = [&](int slot_, int q) {
    if (q >= nrows) return;
    const int jj = q / c.N, nn = q - jj * c.N;
    const unsigned char* src = reinterpret_cast<const unsigned char*>(v) + (size_t)nn * nstride +
                               (size_t)(tok0 + tstride * jj) * RB;
    mbar_arrive_expect_tx(&bar[slot_], (uint32_t)RB);
    bulk_g2s(ring + (size_t)slot_ * RB, src, (uint32_t)RB, &bar[slot_], policy_evict_first());
  };
  if (wk == 0 && lane == 0)
    for (int s = 0; s < c.ring; ++s) issue_row(s, s);
  pdl_trigger();
  if (wtma && !mbar_wait(wbar, 0u)) return;

  const int cb = wk * 256 + lane;  // this lane's chunks: cb + 32k
  const float inv_d = 1.f / (float)c.D;
  int q = 0;
  int ring_slot = 0;  // slot and phase of stream row q (q mod R, (q / R) & 1)
  uint32_t ring_ph = 0;
  for (int j = 0; j < ntok; ++j) {
    float2 o[CPL][P];
#pragma unroll
    for (int k = 0; k < CPL; ++k)
#pragma unroll
      for (int i = 0; i < P; ++i) o[k][i] = make_float2(0.f, 0.f);
    float mref = 0.f, mx = 0.f, l = 0.f;
    float lane_logit = 0.f, lane_r = 0.f;  // row `lane`'s statistics (warp 0 of the stream)
    float* st = stats != nullptr ? stats + (tok0 + tstride * j) * c.stats_stride : nullptr;
    for (int n = 0; n < c.N; ++n, ++q) {
      const int slot = ring_slot;
      const uint32_t ph = ring_ph;
      if (++ring_slot == c.ring) {
        ring_slot = 0;
        ring_ph ^= 1u;
      }
      if (!mbar_wait(&bar[slot], ph)) return;
      const unsigned char* row = ring + (size_t)slot * RB;
      // pass 1: this warp's part of dot and sum of squares
      float2 dacc[2], sacc[2];
#pragma unroll
      for (int a = 0; a < 2; ++a) dacc[a] = sacc[a] = make_float2(0.f, 0.f);
#pragma unroll
      for (int k = 0; k < CPL; ++k) {
        if (k % 4 == 0 && k > 0) __syncwarp();  // bounds the loads hoisted ahead (registers)
        if constexpr (MIX) {
          const uint4 xu = lds128(row + (cb + 32 * k) * 16);
          const uint4 wu = lds128(reinterpret_cast<const unsigned char*>(wsm) + (cb + 32 * k) * 16);
          mixfma2<T>(dacc[0], wu.x, xu.x);
          mixfma2<T>(sacc[0], xu.x, xu.x);
          mixfma2<T>(dacc[1], wu.y, xu.y);
          mixfma2<T>(sacc[1], xu.y, xu.y);
          mixfma2<T>(dacc[0], wu.z, xu.z);
          mixfma2<T>(sacc[0], xu.z, xu.z);
          mixfma2<T>(dacc[1], wu.w, xu.w);
          mixfma2<T>(sacc[1], xu.w, xu.w);
        } else {
          float2 x[P];
          unpack2<T>(lds128(row + (cb + 32 * k) * 16), x);
          const float4* wp = reinterpret_cast<const float4*>(wsm) + (cb + 32 * k);
#pragma unroll
          for (int i = 0; i < P; i += 2) {
            const float4 wv = wp[(i / 2) * RC];
            dacc[0] = __ffma2_rn(make_float2(wv.x, wv.y), x[i], dacc[0]);
            sacc[0] = __ffma2_rn(x[i], x[i], sacc[0]);
            dacc[1] = __ffma2_rn(make_float2(wv.z, wv.w), x[i + 1], dacc[1]);
            sacc[1] = __ffma2_rn(x[i + 1], x[i + 1], sacc[1]);
          }
        }
      }
      dacc[0] = __fadd2_rn(dacc[0], dacc[1]);
      sacc[0] = __fadd2_rn(sacc[0], sacc[1]);
      float2 ds = make_float2(dacc[0].x + dacc[0].y, sacc[0].x + sacc[0].y);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
        ds = __fadd2_rn(ds, make_float2(__shfl_xor_sync(kFull, ds.x, off),
                                        __shfl_xor_sync(kFull, ds.y, off)));
      // the K warps' parts, added in warp order by every warp
      float2* xr = xch + (q & 1) * K;
      if (lane == 0) xr[wk] = ds;
      named_sync(1 + gi, 32 * K);
      ds = xr[0];
#pragma unroll
      for (int k2 = 1; k2 < K; ++k2) ds = __fadd2_rn(ds, xr[k2]);
      const float r = rsqrtf(ds.y * inv_d + c.eps);
      const float logit = ds.x * r;
      if (lane == n) {  // (never for n >= 32: those rows are written directly below)
        lane_logit = logit;
        lane_r = r;
      }
      if (n >= 32 && st != nullptr && wk == 0 && lane == 0) {
        st[n] = logit;
        st[c.N + n] = r;
      }
      constexpr float kRescaleGap = 8.f;
      float wgt = 1.f;
      if (n == 0) {
        mref = mx = logit;
        l = 1.f;
      } else {
        mx = fmaxf(mx, logit);
        if (logit > mref + kRescaleGap) {
          const float sc = expf(mref - logit);
          mref = logit;
          l = fmaf(l, sc, 1.f);
#pragma unroll
          for (int k = 0; k < CPL; ++k)
#pragma unroll
            for (int i = 0; i < P; ++i) o[k][i] = __fmul2_rn(o[k][i], f2(sc));
        } else {
          wgt = expf(logit - mref);
          l += wgt;
        }
      }
      // pass 2: this warp's part of the row again, into o
#pragma unroll
      for (int k = 0; k < CPL; ++k) {
        if (k % 4 == 0 && k > 0) __syncwarp();
        float2 x[P];
        unpack2<T>(lds128(row + (cb + 32 * k) * 16), x);
#pragma unroll
        for (int i = 0; i < P; ++i) o[k][i] = __ffma2_rn(f2(wgt), x[i], o[k][i]);
      }
      // release: the last of the K warps to finish with the buffer refills it
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        if (atomicAdd(&cnt[slot], 1) == K - 1) {
          cnt[slot] = 0;
          __threadfence_block();
          fence_proxy_async();
          issue_row(slot, q + c.ring);
        }
      }
    }
    const long long tok = tok0 + tstride * j;
    if (st != nullptr && wk == 0) {
      if (lane < c.N) {
        st[lane] = lane_logit;
        st[c.N + lane] = lane_r;
      }
      if (lane == 0) {
        st[2 * c.N] = mx;
        st[2 * c.N + 1] = mref + logf(l);
      }
    }
    const float inv = 1.f / l;
    T* orow = out + tok * c.D;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
#pragma unroll
      for (int i = 0; i < P; ++i) o[k][i] = __fmul2_rn(o[k][i], f2(inv));
      stg128(orow + (cb + 32 * k) * VEC, pack2<T>(o[k]));
    }
  }
}

cudaError_t launch_stream_fwd(const StreamCfg& c, int grid, int cpl, int dtype, const void* v,
                              const void* w, int w_dtype, void* out, float* stats, bool sol,
                              cudaStream_t st);

#ifndef SY_TUNE_FWD_MIX
#define SY_TUNE_FWD_MIX 1
#endif

template <typename T, bool FULL, bool MIX>
cudaError_t launch_stream_reread(const StreamCfg& c, int grid, int cpl, dim3 block, size_t smem,
                                 const T* vp, const void* w, int w_dtype, T* op, float* stats,
                                 cudaStream_t st) {
  if (c.kw <= 1 && cpl == 8)
    return launch_smem(stream_fwd_reread_kernel<T, 8, FULL, MIX>, grid, block, smem, st, vp, w,
                       w_dtype, op, stats, c);
  if (c.kw <= 1 && cpl == 4)
    return launch_smem(stream_fwd_reread_kernel<T, 4, FULL, MIX>, grid, block, smem, st, vp, w,
                       w_dtype, op, stats, c);
  if (cpl != 8) return cudaErrorInvalidValue;
  if constexpr (FULL) {
    if (c.kw == 2)
      return launch_smem(stream_fwd_split_kernel<T, 2, MIX>, grid, block, smem, st, vp, w,
                         w_dtype, op, stats, c);
    if (c.kw == 4)
      return launch_smem(stream_fwd_split_kernel<T, 4, MIX>, grid, block, smem, st, vp, w,
                         w_dtype, op, stats, c);
    if (c.kw == 8)
      return launch_smem(stream_fwd_split_kernel<T, 8, MIX>, grid, block, smem, st, vp, w,
                         w_dtype, op, stats, c);
  }
  return cudaErrorInvalidValue;
}

template <typename T, bool SOL, bool FULL>
cudaError_t launch_stream_tf(const StreamCfg& c, int grid, int cpl, const void* v, const void* w,
                             int w_dtype, void* out, float* stats, cudaStream_t st) {
  const size_t smem = stream_smem_layout(c).total;
  const dim3 block(c.warps * 32);
  const T* vp = static_cast<const T*>(v);
  T* op = static_cast<T*>(out);
  if (c.reread) {
    if constexpr (!SOL) {
      if ((cpl == 8 || cpl == 4) && (int)block.x <= kStreamRereadThreads) {
        // w of the sources' own 16-bit type: pass 1 on the packed halves
        if constexpr (sizeof(T) == 2) {
          if (w_dtype == Dt<T>::kCode && SY_TUNE_FWD_MIX)
            return launch_stream_reread<T, FULL, true>(c, grid, cpl, block, smem, vp, w, w_dtype,
                                                       op, stats, st);
        }
        return launch_stream_reread<T, FULL, false>(c, grid, cpl, block, smem, vp, w, w_dtype, op,
                                                    stats, st);
      }
    }
    return cudaErrorInvalidValue;
  }
  switch (cpl) {
    case 1:
      return launch_smem(stream_fwd_kernel<T, 1, SOL, FULL>, grid, block, smem, st, vp, w, w_dtype,
                         op, stats, c);
    case 2:
      return launch_smem(stream_fwd_kernel<T, 2, SOL, FULL>, grid, block, smem, st, vp, w, w_dtype,
                         op, stats, c);
    case 4:
      return launch_smem(stream_fwd_kernel<T, 4, SOL, FULL>, grid, block, smem, st, vp, w, w_dtype,
                         op, stats, c);
    case 8:
      return launch_smem(stream_fwd_kernel<T, 8, SOL, FULL>, grid, block, smem, st, vp, w, w_dtype,
                         op, stats, c);
    default:
      return cudaErrorInvalidValue;
  }
}

template <typename T, bool SOL>
cudaError_t launch_stream_t(const StreamCfg& c, int grid, int cpl, const void* v, const void* w,
                            int w_dtype, void* out, float* stats, cudaStream_t st) {
  if (c.row_chunks == 32 * cpl * (c.kw > 1 ? c.kw : 1))
    return launch_stream_tf<T, SOL, true>(c, grid, cpl, v, w, w_dtype, out, stats, st);
  return launch_stream_tf<T, SOL, false>(c, grid, cpl, v, w, w_dtype, out, stats, st);
}

}  // namespace sy
