// sy_reg.cuh -- "register tile" forward and backward kernels, exact N.
//
// One persistent CTA per SM of G consumer groups x TG threads (no producer
// warp). Group g takes every G-th token of the CTA and owns its own ring of
// S_g shared-memory stages, filled by cp.async.bulk and signalled by one
// mbarrier per stage. The source count N is a compile-time constant (1..16):
//
//  * each thread copies its CPT 16-byte chunks of all N rows from the stage
//    into registers (packed, 4 words per chunk) and does the row reductions
//    on them; once the group has passed its cross-warp barrier every byte of
//    the stage is in registers, and one elected thread immediately refills
//    the stage with the group's token S_g ahead -- the stage is back in flight
//    while the softmax and the weighted sum run from registers;
//  * arithmetic is packed fp32 (fma.rn.f32x2 via __ffma2_rn, two lanes of
//    fp32 per instruction), accumulating even and odd elements separately and
//    adding the pair once per row;
//  * the 2N (forward) or N (backward) row partials are summed across the warp
//    by one reduce-scatter and across the group's warps through shared memory
//    in a fixed order, then every warp redundantly finishes the softmax for
//    its lanes' rows and broadcasts the per-source coefficients with shuffles.
//
// Reference math: src/switchyard/reference.py:42-59 (forward) and the
// derivation in src/switchyard/triton_op.py:205-214 (backward).
#pragma once

#include "sy_launch.cuh"
#include "sy_tile.cuh"

namespace sy {

extern __shared__ __align__(1024) unsigned char sy_smem[];

// Largest N with a register-tile instantiation, and with two- and
// four-chunk ones (the packed tile is N * CPT * 4 registers per thread).
constexpr int kRegMaxN = 16;
constexpr int kRegMaxN2 = 9;   // two chunks per thread up to this N
constexpr int kRegMaxN4 = 6;   // forward: four chunks per thread up to this N
constexpr int kRegFwdMaxN = 9; // forward: larger N takes the row-stream kernel
constexpr int kHoldThreads = 384;        // CTA size of the stage-held forward
constexpr int kHoldMinTokensPerSM = 64;  // use it from this many tokens per SM

#ifndef SY_TUNE_FWD_HOLD
#define SY_TUNE_FWD_HOLD 1  // forward N <= 9: stage-held tile (1) or register tile (0)
#endif

#ifndef SY_TUNE_FWD_UNPACKED_MAX
#define SY_TUNE_FWD_UNPACKED_MAX 144  // largest forward tile kept as fp32 (floats)
#endif
#ifndef SY_TUNE_FWD_PACKED_THREADS
#define SY_TUNE_FWD_PACKED_THREADS 256
#endif

// Forward tile storage: fp32 (unpacked once) when it is small, else the raw
// 16-byte words, unpacked at each use.
__host__ __device__ constexpr bool reg_fwd_packed(int n, int cpt, int vec) {
  return n * cpt * vec > SY_TUNE_FWD_UNPACKED_MAX;
}

// Threads per CTA of a register-tile instantiation (the launch bound that sets
// the register budget): 256, i.e. up to 255 registers per thread.
__host__ __device__ constexpr int reg_threads(int n, int cpt, int vec, bool bwd) {
  return (!bwd && reg_fwd_packed(n, cpt, vec)) ? SY_TUNE_FWD_PACKED_THREADS : 256;
}

// A token's register tile: N rows x CPT chunks, held either as fp32 pairs
// (unpacked once at load) or as the raw 16-byte words (unpacked at each use).
template <typename T, int N, int CPT, bool PACKED>
struct Tile;

template <typename T, int N, int CPT>
struct Tile<T, N, CPT, false> {
  float2 f[N][CPT][Dt<T>::kVec / 2];
  __device__ __forceinline__ void load(int n, int cc, const uint4& u) { unpack2<T>(u, f[n][cc]); }
  __device__ __forceinline__ void get(int n, int cc, float2* p) const {
#pragma unroll
    for (int i = 0; i < Dt<T>::kVec / 2; ++i) p[i] = f[n][cc][i];
  }
};

template <typename T, int N, int CPT>
struct Tile<T, N, CPT, true> {
  uint4 u[N][CPT];
  __device__ __forceinline__ void load(int n, int cc, const uint4& w) { u[n][cc] = w; }
  __device__ __forceinline__ void get(int n, int cc, float2* p) const { unpack2<T>(u[n][cc], p); }
};

// Sum M (16 or 32) per-lane values over the warp. Afterwards lane L holds the
// warp total of value (L >> (5 - log2 M)); for M == 32 that is value L, for
// M == 16 lanes 2i and 2i+1 hold value i. Fixed order, so deterministic and
// bitwise equal in the lanes that share a value.
template <int M>
__device__ __forceinline__ float warp_reduce_scatter(float (&a)[M], int lane) {
  static_assert(M == 16 || M == 32, "M must be 16 or 32");
  if constexpr (M == 32) {
    const bool up = lane & 16;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float send = up ? a[i] : a[i + 16];
      const float keep = up ? a[i + 16] : a[i];
      a[i] = keep + __shfl_xor_sync(kFull, send, 16);
    }
    float b[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) b[i] = a[i];
    // now 16 live values, offsets 8, 4, 2, 1 remain
    {
      const bool u8 = lane & 8;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float send = u8 ? b[i] : b[i + 8];
        const float keep = u8 ? b[i + 8] : b[i];
        b[i] = keep + __shfl_xor_sync(kFull, send, 8);
      }
    }
    {
      const bool u4 = lane & 4;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float send = u4 ? b[i] : b[i + 4];
        const float keep = u4 ? b[i + 4] : b[i];
        b[i] = keep + __shfl_xor_sync(kFull, send, 4);
      }
    }
    {
      const bool u2 = lane & 2;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float send = u2 ? b[i] : b[i + 2];
        const float keep = u2 ? b[i + 2] : b[i];
        b[i] = keep + __shfl_xor_sync(kFull, send, 2);
      }
    }
    const bool u1 = lane & 1;
    const float send = u1 ? b[0] : b[1];
    const float keep = u1 ? b[1] : b[0];
    return keep + __shfl_xor_sync(kFull, send, 1);
  } else {
    return warp_reduce_scatter16(a, lane);
  }
}

// Lane holding value i after warp_reduce_scatter<M>.
template <int M>
__device__ __forceinline__ int rs_src_lane(int i) {
  return M == 32 ? i : 2 * i;
}
template <int M>
__device__ __forceinline__ int rs_index(int lane) {
  return M == 32 ? lane : (lane >> 1);
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
// Per-group ring geometry: group g owns stages [base, base + cnt).
struct GroupRing {
  int base, cnt;
};
__device__ __forceinline__ GroupRing group_ring(int stages, int groups, int g) {
  const int q = stages / groups, rem = stages % groups;
  return {g * q + (g < rem ? g : rem), q + (g < rem ? 1 : 0)};
}

// Issue the bulk copies of one token into a stage: N source rows of
// `row_bytes`, then `extra` optional rows (the backward's g row and the
// token's statistics). One expect_tx covers them all.
__device__ __forceinline__ void issue_token(unsigned char* dst, uint64_t* bar, const unsigned char* vb,
                                            long long tok, int n_rows, int row_bytes,
                                            size_t nstride, const unsigned char* gb,
                                            const float* stats, int stats_bytes,
                                            uint64_t pol) {
  const uint32_t tx = (uint32_t)n_rows * (uint32_t)row_bytes +
                      (gb ? (uint32_t)row_bytes + (uint32_t)stats_bytes : 0u);
  mbar_arrive_expect_tx(bar, tx);
  const unsigned char* src = vb + (size_t)tok * row_bytes;
  for (int n = 0; n < n_rows; ++n)
    bulk_g2s(dst + (size_t)n * row_bytes, src + (size_t)n * nstride, row_bytes, bar, pol);
  if (gb) {
    bulk_g2s(dst + (size_t)n_rows * row_bytes, gb + (size_t)tok * row_bytes, row_bytes, bar, pol);
    bulk_g2s(dst + (size_t)(n_rows + 1) * row_bytes,
             reinterpret_cast<const unsigned char*>(stats) + (size_t)tok * stats_bytes,
             stats_bytes, bar, pol);
  }
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
// HOLD: the tile is not copied to registers; both phases read it from the
// stage, which is refilled only after the group's second barrier (after
// phase B). Far fewer registers per thread, so more groups per CTA.
template <typename T, int N, int CPT, bool HOLD>
__global__ void __launch_bounds__(HOLD ? kHoldThreads : reg_threads(N, CPT, Dt<T>::kVec, false), 1)
    reg_fwd_kernel(const T* __restrict__ v, const void* __restrict__ w, int w_dtype,
                   T* __restrict__ out, float* __restrict__ stats, const TileCfg c) {
  constexpr int VEC = Dt<T>::kVec;
  constexpr int P = VEC / 2;                  // float2 pairs per chunk
  constexpr int M = (2 * N <= 16) ? 16 : 32;  // reduce-scatter width
  constexpr int HALF = M / 2;                 // dot_n at n, ssq_n at HALF + n
  const TileSmem L = tile_smem_layout(c);
  unsigned char* stage0 = sy_smem + L.stages_off;
  float* red_base = reinterpret_cast<float*>(sy_smem + L.red_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(sy_smem + L.bar_off);
  const unsigned char* zero_pad = sy_smem + L.zero_off;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int grid = gridDim.x;
  const int cta = blockIdx.x;
  const int ntok = (cta < c.BT) ? (int)((c.BT - 1 - cta) / grid) + 1 : 0;
  const int wpg = c.tg >> 5;
  const int nwc = c.groups * wpg;

  if (c.N != N || c.groups < 1 || c.stages < c.groups || c.red_stride < M || !c.w_smem) {
    if (tid == 0) record_device_error(kDevErrBadPlan);
    return;
  }
  if (tid == 0) {
    for (int s = 0; s < c.stages; ++s) mbar_init(&full[s], 1);
    *reinterpret_cast<uint4*>(sy_smem + L.zero_off) = make_uint4(0u, 0u, 0u, 0u);
    mbar_fence_init();
  }
  // fp32 w in 16-byte planes: plane q of chunk ch holds w[ch*VEC + 4q .. 4q+3]
  float* wsm = reinterpret_cast<float*>(sy_smem + L.w_off);
  for (int d = tid; d < c.D; d += blockDim.x) {
    const int ch = d / VEC, e = d - ch * VEC;
    wsm[((e >> 2) * c.row_chunks + ch) * 4 + (e & 3)] = load_any(w, w_dtype, d);
  }
  __syncthreads();

  const int g = tid / c.tg;
  const int tig = tid - g * c.tg;
  const int wig = tig >> 5;
  const int cw = tid >> 5;
  const int cw0 = g * wpg;
  const GroupRing ring = group_ring(c.stages, c.groups, g);
  const int ntok_g = ntok > g ? (ntok - 1 - g) / c.groups + 1 : 0;  // this group's tokens
  const uint64_t pol = policy_evict_first();
  const size_t nstride = (size_t)c.BT * c.row_bytes;
  const unsigned char* vb = reinterpret_cast<const unsigned char*>(v);

  // prologue: fill the group's ring
  if (tig == 0)
    for (int j = 0; j < ring.cnt && j < ntok_g; ++j)
      issue_token(stage0 + (size_t)(ring.base + j) * c.stage_bytes, &full[ring.base + j], vb,
                  cta + (long long)(g + j * c.groups) * grid, N, c.row_bytes, nstride, nullptr,
                  nullptr, 0, pol);
  pdl_trigger();  // every CTA is resident: the next kernel may queue for the SMs

  bool cv[CPT];
#pragma unroll
  for (int cc = 0; cc < CPT; ++cc) cv[cc] = tig + cc * c.tg < c.row_chunks;
  const float inv_d = 1.f / (float)c.D;

  int slot = 0;
  uint32_t ph = 0;
  for (int j = 0; j < ntok_g; ++j) {
    const int sidx = ring.base + slot;
    if (!mbar_wait(&full[sidx], ph)) return;
    const unsigned char* tile = stage0 + (size_t)sidx * c.stage_bytes;
    const long long tok = cta + (long long)(g + j * c.groups) * grid;
    // ---- registers <- stage (unpacked once to fp32); phase A ----
    // A chunk past the end of the row reads the 16-byte zero pad instead
    // (stride 0), so the loads need no predicate.
    const unsigned char* cb[CPT];
    int cs[CPT];
#pragma unroll
    for (int cc = 0; cc < CPT; ++cc) {
      cb[cc] = cv[cc] ? tile + (tig + cc * c.tg) * 16 : zero_pad;
      cs[cc] = cv[cc] ? c.row_bytes : 0;
    }
    // The tile stays packed (16-byte words) when unpacking it would not fit
    // the register budget; it is then unpacked again in phase B. In HOLD
    // mode it stays in the stage and is read from there in both phases.
    constexpr bool PACKED = reg_fwd_packed(N, CPT, VEC);
    Tile<T, HOLD ? 1 : N, HOLD ? 1 : CPT, PACKED> x;
    if constexpr (!HOLD) {
#pragma unroll
      for (int n = 0; n < N; ++n)
#pragma unroll
        for (int cc = 0; cc < CPT; ++cc) x.load(n, cc, lds128(cb[cc] + n * cs[cc]));
    }
    auto tget = [&](int n, int cc, float2* p) {
      if constexpr (HOLD)
        unpack2<T>(lds128(cb[cc] + n * cs[cc]), p);
      else
        x.get(n, cc, p);
    };
    // w (fp32, shared memory) for chunk cc, pair i. The load is volatile so
    // the compiler re-reads w per row instead of keeping it in registers,
    // which is the point of the row-outer loop below.
    auto wpair = [&](int cc, int i) {
      const float4* wp = reinterpret_cast<const float4*>(wsm) + (tig + cc * c.tg);
      float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
      if (cv[cc]) q = lds128_f4_volatile(wp + (i / 2) * c.row_chunks);
      return (i & 1) ? make_float2(q.z, q.w) : make_float2(q.x, q.y);
    };
    float a[M];
#pragma unroll
    for (int i = 0; i < M; ++i) a[i] = 0.f;
    if constexpr (PACKED && !HOLD) {
      // row-outer, w re-read per row: two accumulators live instead of 2N
#pragma unroll
      for (int n = 0; n < N; ++n) {
        float2 dot = make_float2(0.f, 0.f), ssq = make_float2(0.f, 0.f);
#pragma unroll
        for (int cc = 0; cc < CPT; ++cc) {
          float2 p[P];
          tget(n, cc, p);
#pragma unroll
          for (int i = 0; i < P; ++i) {
            dot = __ffma2_rn(wpair(cc, i), p[i], dot);
            ssq = __ffma2_rn(p[i], p[i], ssq);
          }
        }
        a[n] = dot.x + dot.y;
        a[HALF + n] = ssq.x + ssq.y;
      }
    } else {
      // chunk-outer: the chunk's w is read once, every row keeps its pairs
      float2 dot2[N], ssq2[N];
#pragma unroll
      for (int n = 0; n < N; ++n) dot2[n] = ssq2[n] = make_float2(0.f, 0.f);
#pragma unroll
      for (int cc = 0; cc < CPT; ++cc) {
        float2 wv[P];
#pragma unroll
        for (int i = 0; i < P; ++i) wv[i] = wpair(cc, i);
#pragma unroll
        for (int n = 0; n < N; ++n) {
          float2 p[P];
          tget(n, cc, p);
#pragma unroll
          for (int i = 0; i < P; ++i) {
            dot2[n] = __ffma2_rn(wv[i], p[i], dot2[n]);
            ssq2[n] = __ffma2_rn(p[i], p[i], ssq2[n]);
          }
        }
      }
#pragma unroll
      for (int n = 0; n < N; ++n) {
        a[n] = dot2[n].x + dot2[n].y;
        a[HALF + n] = ssq2[n].x + ssq2[n].y;
      }
    }
    // ---- cross-thread reduction ----
    const float tot_l = warp_reduce_scatter<M>(a, lane);
    float* red = red_base + (size_t)(j & 1) * nwc * c.red_stride;
    if ((lane & (32 / M - 1)) == 0) red[cw * c.red_stride + rs_index<M>(lane)] = tot_l;
    if (wpg > 1)
      named_sync(1 + g, c.tg);
    else
      __syncwarp();
    // The whole group now holds the stage in registers: refill it with the
    // group's token ring.cnt ahead. (HOLD: after phase B instead.)
    if (!HOLD && tig == 0 && j + ring.cnt < ntok_g) {
      fence_proxy_async();
      issue_token(stage0 + (size_t)sidx * c.stage_bytes, &full[sidx], vb,
                  cta + (long long)(g + (j + ring.cnt) * c.groups) * grid, N, c.row_bytes, nstride,
                  nullptr, nullptr, 0, pol);
    }
    float tot = 0.f;
    for (int q = 0; q < wpg; ++q) tot += red[(cw0 + q) * c.red_stride + rs_index<M>(lane)];

    // ---- softmax over the N sources: lane n < N owns source n ----
    const int ln = lane < N ? lane : 0;
    const float dot = __shfl_sync(kFull, tot, rs_src_lane<M>(ln));
    const float ssq = __shfl_sync(kFull, tot, rs_src_lane<M>(HALF + ln));
    const float r = rsqrtf(ssq * inv_d + c.eps);
    const float logit = lane < N ? dot * r : -INFINITY;
    const float m = warp_max(logit);
    const float e = lane < N ? expf(logit - m) : 0.f;
    const float l = warp_sum(e);
    const float alpha = e / l;
    if (stats != nullptr && wig == 0) {
      float* st = stats + tok * c.stats_stride;
      if (lane < N) {
        st[lane] = logit;
        st[N + lane] = r;
      }
      if (lane == 0) {
        st[2 * N] = m;
        st[2 * N + 1] = m + logf(l);
      }
    }
    float al[N];
#pragma unroll
    for (int n = 0; n < N; ++n) al[n] = __shfl_sync(kFull, alpha, n);

    // ---- phase B: out = sum_n alpha_n v_n from the registers ----
    T* orow = out + tok * c.D;
#pragma unroll
    for (int cc = 0; cc < CPT; ++cc) {
      if (!cv[cc]) continue;
      float2 o[P];
#pragma unroll
      for (int i = 0; i < P; ++i) o[i] = make_float2(0.f, 0.f);
#pragma unroll
      for (int n = 0; n < N; ++n) {
        float2 p[P];
        tget(n, cc, p);
#pragma unroll
        for (int i = 0; i < P; ++i) o[i] = __ffma2_rn(f2(al[n]), p[i], o[i]);
      }
      stg128(orow + (tig + cc * c.tg) * VEC, pack2<T>(o));
    }
    if constexpr (HOLD) {
      // every warp of the group is done with the stage: refill it
      if (wpg > 1)
        named_sync(1 + g, c.tg);
      else
        __syncwarp();
      if (tig == 0 && j + ring.cnt < ntok_g) {
        fence_proxy_async();
        issue_token(stage0 + (size_t)sidx * c.stage_bytes, &full[sidx], vb,
                    cta + (long long)(g + (j + ring.cnt) * c.groups) * grid, N, c.row_bytes,
                    nstride, nullptr, nullptr, 0, pol);
      }
    }

    if (++slot == ring.cnt) {
      slot = 0;
      ph ^= 1u;
    }
  }
}


// ---------------------------------------------------------------------------
// backward (see sy_tile_bwd.cu for the formulas)
// ---------------------------------------------------------------------------
template <typename T, int N, int CPT>
__global__ void __launch_bounds__(reg_threads(N, CPT, Dt<T>::kVec, true), 1)
    reg_bwd_kernel(const T* __restrict__ v, const void* __restrict__ w, int w_dtype,
                   const T* __restrict__ gin, const float* __restrict__ stats, T* __restrict__ dv,
                   float* __restrict__ dw_partial, const TileCfg c) {
  constexpr int VEC = Dt<T>::kVec;
  constexpr int P = VEC / 2;
  constexpr int M = 16;  // N <= 16 partials G_n
  const TileSmem L = tile_smem_layout(c);
  unsigned char* stage0 = sy_smem + L.stages_off;
  float* red_base = reinterpret_cast<float*>(sy_smem + L.red_off);
  float* coef_base = reinterpret_cast<float*>(sy_smem + L.coef_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(sy_smem + L.bar_off);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int grid = gridDim.x;
  const int cta = blockIdx.x;
  const int ntok = (cta < c.BT) ? (int)((c.BT - 1 - cta) / grid) + 1 : 0;
  const int wpg = c.tg >> 5;
  const int nwc = c.groups * wpg;

  if (c.N != N || c.groups < 1 || c.stages < c.groups || c.red_stride < M ||
      c.coef_stride < 4 * N) {
    if (tid == 0) record_device_error(kDevErrBadPlan);
    return;
  }
  if (tid == 0) {
    for (int s = 0; s < c.stages; ++s) mbar_init(&full[s], 1);
    mbar_fence_init();
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
  const unsigned char* gb = reinterpret_cast<const unsigned char*>(gin);
  const int st_bytes = c.stats_stride * 4;

  // Launched as a programmatic dependent of the forward: its inputs are
  // read only after that kernel has completed.
  pdl_wait();
  // w's loads go out before the ring fill (issued after it, they would wait
  // behind the bulk copies); they are first needed in phase B.
  bool cv[CPT];
  float2 w2[CPT][P], dw2[CPT][P];
#pragma unroll
  for (int cc = 0; cc < CPT; ++cc) {
    const int chunk = tig + cc * c.tg;
    cv[cc] = chunk < c.row_chunks;
#pragma unroll
    for (int i = 0; i < P; ++i) {
      w2[cc][i] = cv[cc] ? make_float2(load_any(w, w_dtype, (long long)chunk * VEC + 2 * i),
                                       load_any(w, w_dtype, (long long)chunk * VEC + 2 * i + 1))
                         : make_float2(0.f, 0.f);
      dw2[cc][i] = make_float2(0.f, 0.f);
    }
  }
  const float inv_d = 1.f / (float)c.D;

  if (tig == 0)
    for (int j = 0; j < ring.cnt && j < ntok_g; ++j)
      issue_token(stage0 + (size_t)(ring.base + j) * c.stage_bytes, &full[ring.base + j], vb,
                  cta + (long long)(g + j * c.groups) * grid, N, c.row_bytes, nstride, gb, stats,
                  st_bytes, pol);

  int slot = 0;
  uint32_t ph = 0;
  bool ok = true;
  for (int j = 0; j < ntok_g; ++j) {
    const int sidx = ring.base + slot;
    if (!mbar_wait(&full[sidx], ph)) {
      ok = false;
      break;
    }
    const unsigned char* tile = stage0 + (size_t)sidx * c.stage_bytes;
    const float* st = reinterpret_cast<const float*>(tile + (size_t)(N + 1) * c.row_bytes);
    const long long tok = cta + (long long)(g + j * c.groups) * grid;

    uint4 x[N][CPT], gx[CPT];
#pragma unroll
    for (int n = 0; n < N; ++n)
#pragma unroll
      for (int cc = 0; cc < CPT; ++cc)
        x[n][cc] = cv[cc] ? lds128(tile + (size_t)n * c.row_bytes + (tig + cc * c.tg) * 16)
                          : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int cc = 0; cc < CPT; ++cc)
      gx[cc] = cv[cc] ? lds128(tile + (size_t)N * c.row_bytes + (tig + cc * c.tg) * 16)
                      : make_uint4(0u, 0u, 0u, 0u);
    // lane n < N keeps its source's saved logit and inverse RMS
    const int ln = lane < N ? lane : 0;
    const float logit = st[ln];
    const float r = st[N + ln];
    const float alpha = lane < N ? expf(logit - st[2 * N + 1]) : 0.f;

    // ---- phase A: G_n = g . v_n ----
    float a[M];
#pragma unroll
    for (int i = 0; i < M; ++i) a[i] = 0.f;
#pragma unroll
    for (int cc = 0; cc < CPT; ++cc) {
      if constexpr (sizeof(T) == 2) {
        // packed 16-bit halves, word i = pair i: the same products and order
        // as the unpacked form below, without unpacking the tile
#pragma unroll
        for (int n = 0; n < N; ++n) {
          float2 acc = make_float2(0.f, 0.f);
          mixfma2<T>(acc, gx[cc].x, x[n][cc].x);
          mixfma2<T>(acc, gx[cc].y, x[n][cc].y);
          mixfma2<T>(acc, gx[cc].z, x[n][cc].z);
          mixfma2<T>(acc, gx[cc].w, x[n][cc].w);
          a[n] += acc.x + acc.y;
        }
      } else {
        float2 gp[P];
        unpack2<T>(gx[cc], gp);
#pragma unroll
        for (int n = 0; n < N; ++n) {
          float2 p[P];
          unpack2<T>(x[n][cc], p);
          float2 acc = make_float2(0.f, 0.f);
#pragma unroll
          for (int i = 0; i < P; ++i) acc = __ffma2_rn(gp[i], p[i], acc);
          a[n] += acc.x + acc.y;
        }
      }
    }
    const float tot_l = warp_reduce_scatter<M>(a, lane);
    float* red = red_base + (size_t)(j & 1) * nwc * c.red_stride;
    if ((lane & 1) == 0) red[cw * c.red_stride + (lane >> 1)] = tot_l;
    if (wpg > 1)
      named_sync(1 + g, c.tg);
    else
      __syncwarp();
    if (tig == 0 && j + ring.cnt < ntok_g) {
      fence_proxy_async();
      issue_token(stage0 + (size_t)sidx * c.stage_bytes, &full[sidx], vb,
                  cta + (long long)(g + (j + ring.cnt) * c.groups) * grid, N, c.row_bytes, nstride,
                  gb, stats, st_bytes, pol);
    }
    float tot = 0.f;
    for (int q = 0; q < wpg; ++q) tot += red[(cw0 + q) * c.red_stride + (lane >> 1)];

    // ---- per-source coefficients: lane n < N owns source n ----
    const float Gn = __shfl_sync(kFull, tot, 2 * ln);
    const float S = warp_sum(lane < N ? alpha * Gn : 0.f);
    const float dl = alpha * (Gn - S);
    const float da_l = dl * r;
    const float cv_l = -dl * logit * r * r * inv_d;
    // The warp's coefficients go to its own slot of shared memory and are
    // read back with broadcast loads (cheaper in registers than 3N shuffles).
    float4* coef = reinterpret_cast<float4*>(coef_base + (size_t)cw * c.coef_stride);
    __syncwarp();  // the previous token's phase B reads of coef are done
    if (lane < N) coef[lane] = make_float4(alpha, da_l, cv_l, 0.f);
    __syncwarp();

    // ---- phase B: dv_n = alpha_n g + da_n w + cv_n v_n ; dw += da_n v_n ----
#pragma unroll
    for (int cc = 0; cc < CPT; ++cc) {
      if (!cv[cc]) continue;
      float2 gp[P];
      unpack2<T>(gx[cc], gp);
      T* dcol = dv + (size_t)tok * c.D + (size_t)(tig + cc * c.tg) * VEC;
#pragma unroll
      for (int n = 0; n < N; ++n) {
        const float4 k = coef[n];  // alpha, da, cv
        float2 p[P], d[P];
        unpack2<T>(x[n][cc], p);
#pragma unroll
        for (int i = 0; i < P; ++i) {
          d[i] = __ffma2_rn(f2(k.z), p[i], __ffma2_rn(f2(k.y), w2[cc][i], __fmul2_rn(f2(k.x), gp[i])));
          dw2[cc][i] = __ffma2_rn(f2(k.y), p[i], dw2[cc][i]);
        }
        stg128(dcol + (size_t)n * c.BT * c.D, pack2<T>(d));
      }
    }

    if (++slot == ring.cnt) {
      slot = 0;
      ph ^= 1u;
    }
  }

  // ---- one dw partial row per CTA: the groups' accumulators are added in
  // group order through shared memory (the stages are idle by now) ----
  // (CTA-uniform: if any group's wait ran out, every thread leaves here.)
  if (!__syncthreads_and(ok)) return;
  float* acc = reinterpret_cast<float*>(stage0);  // [groups][D] fp32
#pragma unroll
  for (int cc = 0; cc < CPT; ++cc) {
    if (!cv[cc]) continue;
    float* dst = acc + (size_t)g * c.D + (size_t)(tig + cc * c.tg) * VEC;
#pragma unroll
    for (int i = 0; i < P; i += 2)
      *reinterpret_cast<float4*>(dst + 2 * i) =
          make_float4(dw2[cc][i].x, dw2[cc][i].y, dw2[cc][i + 1].x, dw2[cc][i + 1].y);
  }
  __syncthreads();
  float* prow = dw_partial + (size_t)cta * c.D;
  for (int d = tid * 4; d < c.D; d += blockDim.x * 4) {
    float4 t = *reinterpret_cast<const float4*>(acc + d);
    for (int q = 1; q < c.groups; ++q) {
      const float4 u = *reinterpret_cast<const float4*>(acc + (size_t)q * c.D + d);
      t.x += u.x;
      t.y += u.y;
      t.z += u.z;
      t.w += u.w;
    }
    *reinterpret_cast<float4*>(prow + d) = t;
  }
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// launchers: dispatch the run-time N and CPT onto the instantiations
// ---------------------------------------------------------------------------
template <typename T, int N>
cudaError_t launch_reg_fwd_n(const TileCfg& c, int grid, int cpt, const void* v, const void* w,
                             int w_dtype, void* out, float* stats, cudaStream_t st) {
  const size_t smem = tile_smem_layout(c).total;
  const dim3 block(c.groups * c.tg);  // no producer warp
  const T* vp = static_cast<const T*>(v);
  T* op = static_cast<T*>(out);
  if (c.hold) {
    if ((int)block.x > kHoldThreads) return cudaErrorInvalidConfiguration;
    if constexpr (N <= kRegFwdMaxN) {
      if (cpt == 4)
        return launch_smem(reg_fwd_kernel<T, N, 4, true>, grid, block, smem, st, vp, w, w_dtype,
                           op, stats, c);
      if (cpt == 2)
        return launch_smem(reg_fwd_kernel<T, N, 2, true>, grid, block, smem, st, vp, w, w_dtype,
                           op, stats, c);
      if (cpt == 1)
        return launch_smem(reg_fwd_kernel<T, N, 1, true>, grid, block, smem, st, vp, w, w_dtype,
                           op, stats, c);
    }
    return cudaErrorInvalidValue;
  }
  if ((int)block.x > reg_threads(N, cpt, Dt<T>::kVec, false)) return cudaErrorInvalidConfiguration;
  if (cpt == 1)
    return launch_smem(reg_fwd_kernel<T, N, 1, false>, grid, block, smem, st, vp, w, w_dtype, op,
                       stats, c);
  if constexpr (N <= kRegMaxN2)
    if (cpt == 2)
      return launch_smem(reg_fwd_kernel<T, N, 2, false>, grid, block, smem, st, vp, w, w_dtype, op,
                         stats, c);
  if constexpr (N <= kRegMaxN4)
    if (cpt == 4)
      return launch_smem(reg_fwd_kernel<T, N, 4, false>, grid, block, smem, st, vp, w, w_dtype, op,
                         stats, c);
  return cudaErrorInvalidValue;
}

template <typename T, int N>
cudaError_t launch_reg_bwd_n(const TileCfg& c, int grid, int cpt, const void* v, const void* w,
                             int w_dtype, const void* g, const float* stats, void* dv, float* dwp,
                             cudaStream_t st) {
  const size_t smem = tile_smem_layout(c).total;
  const dim3 block(c.groups * c.tg);  // no producer warp
  if ((int)block.x > reg_threads(N, cpt, Dt<T>::kVec, true)) return cudaErrorInvalidConfiguration;
  const T* vp = static_cast<const T*>(v);
  const T* gp = static_cast<const T*>(g);
  T* dvp = static_cast<T*>(dv);
  if (cpt == 1)
    return launch_smem_pdl(reg_bwd_kernel<T, N, 1>, grid, block, smem, st, vp, w, w_dtype, gp, stats,
                       dvp, dwp, c);
  if constexpr (N <= kRegMaxN2)
    if (cpt == 2)
      return launch_smem_pdl(reg_bwd_kernel<T, N, 2>, grid, block, smem, st, vp, w, w_dtype, gp, stats,
                         dvp, dwp, c);
  return cudaErrorInvalidValue;
}

#define SY_REG_CASES(F, ...) \
  case 1: return F<T, 1>(__VA_ARGS__);   \
  case 2: return F<T, 2>(__VA_ARGS__);   \
  case 3: return F<T, 3>(__VA_ARGS__);   \
  case 4: return F<T, 4>(__VA_ARGS__);   \
  case 5: return F<T, 5>(__VA_ARGS__);   \
  case 6: return F<T, 6>(__VA_ARGS__);   \
  case 7: return F<T, 7>(__VA_ARGS__);   \
  case 8: return F<T, 8>(__VA_ARGS__);   \
  case 9: return F<T, 9>(__VA_ARGS__);   \
  case 10: return F<T, 10>(__VA_ARGS__); \
  case 11: return F<T, 11>(__VA_ARGS__); \
  case 12: return F<T, 12>(__VA_ARGS__); \
  case 13: return F<T, 13>(__VA_ARGS__); \
  case 14: return F<T, 14>(__VA_ARGS__); \
  case 15: return F<T, 15>(__VA_ARGS__); \
  case 16: return F<T, 16>(__VA_ARGS__);

template <typename T>
cudaError_t launch_reg_fwd_t(const TileCfg& c, int grid, int cpt, const void* v, const void* w,
                             int w_dtype, void* out, float* stats, cudaStream_t st) {
  switch (c.N) {
    SY_REG_CASES(launch_reg_fwd_n, c, grid, cpt, v, w, w_dtype, out, stats, st)
    default:
      return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t launch_reg_bwd_t(const TileCfg& c, int grid, int cpt, const void* v, const void* w,
                             int w_dtype, const void* g, const float* stats, void* dv, float* dwp,
                             cudaStream_t st) {
  switch (c.N) {
    SY_REG_CASES(launch_reg_bwd_n, c, grid, cpt, v, w, w_dtype, g, stats, dv, dwp, st)
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace sy
