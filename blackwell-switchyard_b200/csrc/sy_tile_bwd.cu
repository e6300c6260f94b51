// sy_tile_bwd.cu -- backward tile kernel and the fixed-order dw reduction.
//
// Backward, per token, from the statistics the forward saved
// (logit_n, r_n = 1/rms_n, lse). With G_n = g.v_n and S = sum_n alpha_n G_n:
//   alpha_n  = exp(logit_n - lse)
//   dlogit_n = alpha_n (G_n - S)                 softmax backward
//   da_n     = dlogit_n r_n                      through logit = a r
//   2 dssq_n = -dlogit_n logit_n r_n^2 / D       through r = (ssq/D+eps)^-1/2
//   dv_n     = alpha_n g + da_n w + 2 dssq_n v_n
//   dw      += sum_n da_n v_n                    (per consumer group, fp32)
// Same derivation as the reference kernel's docstring
// (src/switchyard/triton_op.py:205-214); the reference recomputes ssq and a
// from v, this kernel reads them back from the saved logit and r.
//
// Stage contents: N rows of v, one row of g, the token's statistics row. Only
// G_n needs a cross-thread reduction (16 rows per reduce-scatter). Every
// consumer group owns one fp32 row of dw_partial and accumulates its tokens
// into registers in token order; sy_dw_reduce sums the rows in a fixed order,
// so dw is deterministic and needs no atomics and no zero-fill.
#include "sy_launch.cuh"
#include "sy_tile.cuh"

namespace sy {

extern __shared__ __align__(1024) unsigned char sy_smem[];

template <typename T, int CPT>
__global__ void __launch_bounds__(32 + kConsumerThreads, 1)
    tile_bwd_kernel(const T* __restrict__ v, const void* __restrict__ w, int w_dtype,
                    const T* __restrict__ gin, const float* __restrict__ stats, T* __restrict__ dv,
                    float* __restrict__ dw_partial, const TileCfg c) {
  constexpr int VEC = Dt<T>::kVec;
  const TileSmem L = tile_smem_layout(c);
  unsigned char* stage0 = sy_smem + L.stages_off;
  float* red_base = reinterpret_cast<float*>(sy_smem + L.red_off);
  float* coef_base = reinterpret_cast<float*>(sy_smem + L.coef_off);
  uint64_t* full = reinterpret_cast<uint64_t*>(sy_smem + L.bar_off);
  uint64_t* empty = full + c.stages;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int grid = gridDim.x;
  const int cta = blockIdx.x;
  const int ntok = (cta < c.BT) ? (int)((c.BT - 1 - cta) / grid) + 1 : 0;
  const int wpg = c.tg >> 5;
  const int nwc = c.groups * wpg;
  const int N = c.N;

  // The stage/group protocol needs S % G == 0 (see the planner); refuse any
  // other plan instead of running it.
  if (c.groups < 1 || c.stages % c.groups != 0) {
    if (tid == 0) record_device_error(kDevErrBadPlan);
    return;
  }
  if (tid == 0) {
    for (int s = 0; s < c.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], wpg);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const uint32_t st_bytes = (uint32_t)c.stats_stride * 4u;
      const uint32_t tx = (uint32_t)(N + 1) * (uint32_t)c.row_bytes + st_bytes;
      const size_t nstride = (size_t)c.BT * c.row_bytes;
      const unsigned char* vb = reinterpret_cast<const unsigned char*>(v);
      const unsigned char* gb = reinterpret_cast<const unsigned char*>(gin);
      int s = 0;
      uint32_t ph = 0;
      for (int k = 0; k < ntok; ++k) {
        if (!mbar_wait(&empty[s], ph ^ 1u)) break;
        const long long tok = cta + (long long)k * grid;
        unsigned char* dst = stage0 + (size_t)s * c.stage_bytes;
        mbar_arrive_expect_tx(&full[s], tx);
        const unsigned char* src = vb + (size_t)tok * c.row_bytes;
        for (int n = 0; n < N; ++n)
          bulk_g2s(dst + (size_t)n * c.row_bytes, src + (size_t)n * nstride, c.row_bytes, &full[s],
                   pol);
        bulk_g2s(dst + (size_t)N * c.row_bytes, gb + (size_t)tok * c.row_bytes, c.row_bytes,
                 &full[s], pol);
        bulk_g2s(dst + (size_t)(N + 1) * c.row_bytes, stats + (size_t)tok * c.stats_stride,
                 st_bytes, &full[s], pol);
        if (++s == c.stages) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
    return;
  }

  const int ct = tid - 32;
  const int g = ct / c.tg;
  const int tig = ct - g * c.tg;
  const int cw = ct >> 5;
  const int cw0 = g * wpg;

  float wr[CPT][VEC], dwacc[CPT][VEC];
#pragma unroll
  for (int cc = 0; cc < CPT; ++cc) {
    const int chunk = tig + cc * c.tg;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      wr[cc][e] = (chunk < c.row_chunks) ? load_any(w, w_dtype, (long long)chunk * VEC + e) : 0.f;
      dwacc[cc][e] = 0.f;
    }
  }
  float4* coef = reinterpret_cast<float4*>(coef_base + (size_t)cw * c.coef_stride);
  const float inv_d = 1.f / (float)c.D;

  int s = g % c.stages;
  uint32_t ph = (uint32_t)((g / c.stages) & 1);
  int it = 0;
  bool ok = true;
  for (int k = g; k < ntok; k += c.groups, ++it) {
    if (!mbar_wait(&full[s], ph)) {
      ok = false;
      break;
    }
    const unsigned char* tile = stage0 + (size_t)s * c.stage_bytes;
    const float* st = reinterpret_cast<const float*>(tile + (size_t)(N + 1) * c.row_bytes);
    const long long tok = cta + (long long)k * grid;

    float gr[CPT][VEC];
#pragma unroll
    for (int cc = 0; cc < CPT; ++cc) {
      const int chunk = tig + cc * c.tg;
      if (chunk < c.row_chunks) {
        Dt<T>::unpack(lds128(tile + (size_t)N * c.row_bytes + chunk * 16), gr[cc]);
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) gr[cc][e] = 0.f;
      }
    }

    // ---- phase A: G_n = g . v_n, 16 rows per reduce-scatter ----
    const int buf = it & 1;
    float* red_w = red_base + ((size_t)buf * nwc + cw) * c.red_stride;
    for (int b16 = 0; b16 * 16 < N; ++b16) {
      float a[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) a[i] = 0.f;
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        const int n = b16 * 16 + r;
        if (n < N) {
          const unsigned char* row = tile + (size_t)n * c.row_bytes;
#pragma unroll
          for (int cc = 0; cc < CPT; ++cc) {
            const int chunk = tig + cc * c.tg;
            if (chunk < c.row_chunks) {
              float x[VEC];
              Dt<T>::unpack(lds128(row + chunk * 16), x);
#pragma unroll
              for (int e = 0; e < VEC; ++e) a[r] = fmaf(gr[cc][e], x[e], a[r]);
            }
          }
        }
      }
      const float tot = warp_reduce_scatter16(a, lane);
      if ((lane & 1) == 0) red_w[b16 * 16 + (lane >> 1)] = tot;
    }
    if (wpg > 1)
      named_sync(1 + g, c.tg);
    else
      __syncwarp();

    // ---- per-source coefficients: lane j owns rows j and j+32 ----
    const float* red_g = red_base + ((size_t)buf * nwc + cw0) * c.red_stride;
    const float lse = st[2 * N + 1];
    float al[2], Gn[2], lg[2], rr[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int n = lane + 32 * j;
      al[j] = 0.f;
      Gn[j] = 0.f;
      lg[j] = 0.f;
      rr[j] = 0.f;
      if (n < N) {
        const int off = (n >> 4) * 16 + (n & 15);
        float gs = 0.f;
        for (int q = 0; q < wpg; ++q) gs += red_g[q * c.red_stride + off];
        Gn[j] = gs;
        lg[j] = st[n];
        rr[j] = st[N + n];
        al[j] = expf(lg[j] - lse);
      }
    }
    const float S = warp_sum(al[0] * Gn[0] + al[1] * Gn[1]);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int n = lane + 32 * j;
      if (n < N) {
        const float dl = al[j] * (Gn[j] - S);
        const float da = dl * rr[j];
        const float cv = -dl * lg[j] * rr[j] * rr[j] * inv_d;
        coef[n] = make_float4(al[j], da, cv, 0.f);
      }
    }
    __syncwarp();

    // ---- phase B: dv rows and the dw accumulation ----
#pragma unroll
    for (int cc = 0; cc < CPT; ++cc) {
      const int chunk = tig + cc * c.tg;
      if (chunk < c.row_chunks) {
        for (int n = 0; n < N; ++n) {
          const float4 cf = coef[n];
          float x[VEC], d[VEC];
          Dt<T>::unpack(lds128(tile + (size_t)n * c.row_bytes + chunk * 16), x);
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            d[e] = fmaf(cf.z, x[e], fmaf(cf.y, wr[cc][e], cf.x * gr[cc][e]));
            dwacc[cc][e] = fmaf(cf.y, x[e], dwacc[cc][e]);
          }
          stg128(dv + ((size_t)n * c.BT + tok) * c.D + (size_t)chunk * VEC, Dt<T>::pack(d));
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    s += c.groups;
    while (s >= c.stages) {
      s -= c.stages;
      ph ^= 1u;
    }
  }

  // ---- this group's dw partial row (written even when it saw no token) ----
  if (ok) {
    float* prow = dw_partial + ((size_t)cta * c.groups + g) * c.D;
#pragma unroll
    for (int cc = 0; cc < CPT; ++cc) {
      const int chunk = tig + cc * c.tg;
      if (chunk < c.row_chunks) {
#pragma unroll
        for (int e = 0; e < VEC; e += 4)
          *reinterpret_cast<float4*>(prow + (size_t)chunk * VEC + e) =
              make_float4(dwacc[cc][e], dwacc[cc][e + 1], dwacc[cc][e + 2], dwacc[cc][e + 3]);
      }
    }
  }
  // Let the dependent dw reduction launch; it still waits for this grid to
  // complete before reading the partials.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename T>
static cudaError_t launch_bwd_t(const TileCfg& c, int grid, int cpt, const void* v, const void* w,
                                int w_dtype, const void* g, const float* stats, void* dv,
                                float* dwp, cudaStream_t st) {
  const size_t smem = tile_smem_layout(c).total;
  const dim3 block(32 + c.groups * c.tg);
  const T* vp = static_cast<const T*>(v);
  const T* gp = static_cast<const T*>(g);
  T* dvp = static_cast<T*>(dv);
  switch (cpt) {
    case 1:
      return launch_smem(tile_bwd_kernel<T, 1>, grid, block, smem, st, vp, w, w_dtype, gp, stats,
                         dvp, dwp, c);
    case 2:
      return launch_smem(tile_bwd_kernel<T, 2>, grid, block, smem, st, vp, w, w_dtype, gp, stats,
                         dvp, dwp, c);
    case 4:
      return launch_smem(tile_bwd_kernel<T, 4>, grid, block, smem, st, vp, w, w_dtype, gp, stats,
                         dvp, dwp, c);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_tile_bwd(const TileCfg& c, int grid, int cpt, int dtype, const void* v,
                            const void* w, int w_dtype, const void* g, const float* stats,
                            void* dv, float* dw_partial, cudaStream_t st) {
  switch (dtype) {
    case SY_BF16:
      return launch_bwd_t<__nv_bfloat16>(c, grid, cpt, v, w, w_dtype, g, stats, dv, dw_partial, st);
    case SY_F16:
      return launch_bwd_t<__half>(c, grid, cpt, v, w, w_dtype, g, stats, dv, dw_partial, st);
    case SY_F32:
      return launch_bwd_t<float>(c, grid, cpt, v, w, w_dtype, g, stats, dv, dw_partial, st);
    default:
      return cudaErrorInvalidValue;
  }
}

// ---------------------------------------------------------------------------
// dw[d] = sum_p part[p, d]. A CTA owns 32 consecutive columns; warp k of its 8
// sums rows p = k, k+8, k+16, ... in increasing order (loaded 32 at a time),
// then warp 0 adds the 8 warp sums in warp order. Fixed order everywhere =>
// deterministic.
// With a gain (gw, gg non-null) the sum is the gradient of q = w * g: it is
// rounded to dw_dtype (as the plain reduction stores it) and split into
// dw = dq * g and dg = dq * w, each rounded to dw_dtype -- the products and
// roundings of the two elementwise autograd kernels it replaces. dw or dg
// may be null (no gradient wanted).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float round_as(int dtype, float x) {
  switch (dtype) {
    case SY_BF16:
      return __bfloat162float(__float2bfloat16_rn(x));
    case SY_F16:
      return __half2float(__float2half_rn(x));
    default:
      return x;
  }
}

__global__ void __launch_bounds__(256) dw_reduce_kernel(const float* __restrict__ part, long long P,
                                                        long long D, void* __restrict__ dw,
                                                        int dw_dtype, const void* __restrict__ gw,
                                                        const void* __restrict__ gg,
                                                        void* __restrict__ dg) {
  __shared__ float slice[8][33];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const int wp = threadIdx.x >> 5;
  const long long col = (long long)blockIdx.x * 32 + lane;
  // all of a batch's loads are issued before the first add: one DRAM round
  // trip per 32 rows instead of one per row
  const float acc = col < D ? partial_rows_warp_sum(part, P, D, col, wp) : 0.f;
  slice[wp][lane] = acc;
  __syncthreads();
  if (wp == 0 && col < D) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += slice[i][lane];
    if (gg == nullptr) {
      store_any(dw, dw_dtype, col, t);
    } else {
      const float dq = round_as(dw_dtype, t);
      if (dw) store_any(dw, dw_dtype, col, dq * load_any(gg, dw_dtype, col));
      if (dg) store_any(dg, dw_dtype, col, dq * load_any(gw, dw_dtype, col));
    }
  }
}

cudaError_t launch_dw_reduce(const float* part, long long P, long long D, void* dw, int dw_dtype,
                             bool pdl, cudaStream_t st, const void* gw, const void* gg, void* dg) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((D + 31) / 32));
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, dw_reduce_kernel, part, P, D, dw, dw_dtype, gw, gg, dg);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace sy
