// sy_tile_fwd.cu -- forward and speed-of-light tile kernels (sm_100a).
//
// Forward, per token (reference math: src/switchyard/reference.py:42-59; the
// Triton kernels it replaces: src/switchyard/triton_op.py:50-117):
//   phase A  every consumer thread accumulates dot_n = w.v_n and
//            ssq_n = v_n.v_n over its chunks, eight rows at a time; the 16
//            partials are summed across the warp by one reduce-scatter and
//            across the group's warps through shared memory.
//   softmax  each warp (redundantly, so no second barrier) computes
//            logit_n = dot_n * rsqrt(ssq_n/D + eps), the max, the exp-sum and
//            alpha_n for its lane's rows, and keeps alpha in a per-warp
//            shared array; warp 0 of the group writes the token's statistics.
//   phase B  out = sum_n alpha_n v_n over the thread's chunks, from the same
//            shared-memory tile, rounded once to the output dtype.
// All arithmetic is fp32; v is read from HBM once.
#include "sy_tile.cuh"
#include "sy_launch.cuh"

namespace sy {

extern __shared__ __align__(1024) unsigned char sy_smem[];

template <typename T, int CPT, bool SOL>
__global__ void __launch_bounds__(32 + kConsumerThreads, 1)
    tile_fwd_kernel(const T* __restrict__ v, const void* __restrict__ w, int w_dtype,
                    T* __restrict__ out, float* __restrict__ stats, const TileCfg c) {
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
  const int wpg = c.tg >> 5;  // warps per consumer group
  const int nwc = c.groups * wpg;

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
    // ---------------- producer: one lane streams rows into the ring ----------
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const uint32_t tx = (uint32_t)c.N * (uint32_t)c.row_bytes;
      const size_t nstride = (size_t)c.BT * c.row_bytes;
      const unsigned char* vb = reinterpret_cast<const unsigned char*>(v);
      int s = 0;
      uint32_t ph = 0;
      for (int k = 0; k < ntok; ++k) {
        if (!mbar_wait(&empty[s], ph ^ 1u)) break;
        const long long tok = cta + (long long)k * grid;
        unsigned char* dst = stage0 + (size_t)s * c.stage_bytes;
        const unsigned char* src = vb + (size_t)tok * c.row_bytes;
        mbar_arrive_expect_tx(&full[s], tx);
        for (int n = 0; n < c.N; ++n)
          bulk_g2s(dst + (size_t)n * c.row_bytes, src + (size_t)n * nstride, c.row_bytes, &full[s],
                   pol);
        if (++s == c.stages) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
    return;
  }

  // ---------------- consumers -------------------------------------------------
  const int ct = tid - 32;
  const int g = ct / c.tg;
  const int tig = ct - g * c.tg;
  const int wig = tig >> 5;  // warp index within the group
  const int cw = ct >> 5;    // consumer warp index within the CTA
  const int cw0 = g * wpg;

  float wr[CPT][VEC];
  if constexpr (!SOL) {
#pragma unroll
    for (int cc = 0; cc < CPT; ++cc) {
      const int chunk = tig + cc * c.tg;
#pragma unroll
      for (int e = 0; e < VEC; ++e)
        wr[cc][e] = (chunk < c.row_chunks) ? load_any(w, w_dtype, (long long)chunk * VEC + e) : 0.f;
    }
  }
  float* alpha = coef_base + (size_t)cw * c.coef_stride;

  int s = g % c.stages;
  uint32_t ph = (uint32_t)((g / c.stages) & 1);
  int it = 0;  // this group's iteration count (selects the reduction buffer)
  for (int k = g; k < ntok; k += c.groups, ++it) {
    if (!mbar_wait(&full[s], ph)) return;
    const unsigned char* tile = stage0 + (size_t)s * c.stage_bytes;
    const long long tok = cta + (long long)k * grid;
    T* orow = out + tok * c.D;

    if constexpr (SOL) {
#pragma unroll
      for (int cc = 0; cc < CPT; ++cc) {
        const int chunk = tig + cc * c.tg;
        if (chunk < c.row_chunks) {
          float o[VEC];
#pragma unroll
          for (int e = 0; e < VEC; ++e) o[e] = 0.f;
          for (int n = 0; n < c.N; ++n) {
            float x[VEC];
            Dt<T>::unpack(lds128(tile + (size_t)n * c.row_bytes + chunk * 16), x);
#pragma unroll
            for (int e = 0; e < VEC; ++e) o[e] += x[e];
          }
          stg128(orow + chunk * VEC, Dt<T>::pack(o));
        }
      }
    } else {
      // ---- phase A: dot and sum of squares, 8 rows per reduce-scatter ----
      const int buf = it & 1;
      float* red_w = red_base + ((size_t)buf * nwc + cw) * c.red_stride;
      for (int b8 = 0; b8 * 8 < c.N; ++b8) {
        float a[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) a[i] = 0.f;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const int n = b8 * 8 + r;
          if (n < c.N) {
            const unsigned char* row = tile + (size_t)n * c.row_bytes;
#pragma unroll
            for (int cc = 0; cc < CPT; ++cc) {
              const int chunk = tig + cc * c.tg;
              if (chunk < c.row_chunks) {
                float x[VEC];
                Dt<T>::unpack(lds128(row + chunk * 16), x);
#pragma unroll
                for (int e = 0; e < VEC; ++e) {
                  a[r] = fmaf(wr[cc][e], x[e], a[r]);
                  a[8 + r] = fmaf(x[e], x[e], a[8 + r]);
                }
              }
            }
          }
        }
        const float tot = warp_reduce_scatter16(a, lane);
        if ((lane & 1) == 0) red_w[b8 * 16 + (lane >> 1)] = tot;
      }
      if (wpg > 1)
        named_sync(1 + g, c.tg);
      else
        __syncwarp();

      // ---- softmax over sources: lane j owns rows j and j+32 ----
      const float* red_g = red_base + ((size_t)buf * nwc + cw0) * c.red_stride;
      float lg[2], rr[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int n = lane + 32 * j;
        lg[j] = -INFINITY;
        rr[j] = 0.f;
        if (n < c.N) {
          const int off = (n >> 3) * 16 + (n & 7);
          float dot = 0.f, ssq = 0.f;
          for (int q = 0; q < wpg; ++q) {
            dot += red_g[q * c.red_stride + off];
            ssq += red_g[q * c.red_stride + off + 8];
          }
          rr[j] = rsqrtf(ssq / (float)c.D + c.eps);
          lg[j] = dot * rr[j];
        }
      }
      const float m = warp_max(fmaxf(lg[0], lg[1]));
      const float p0 = (lane < c.N) ? expf(lg[0] - m) : 0.f;
      const float p1 = (lane + 32 < c.N) ? expf(lg[1] - m) : 0.f;
      const float l = warp_sum(p0 + p1);
      const float inv = 1.f / l;
      if (lane < c.N) alpha[lane] = p0 * inv;
      if (lane + 32 < c.N) alpha[lane + 32] = p1 * inv;
      if (stats != nullptr && wig == 0) {
        float* st = stats + tok * c.stats_stride;
        if (lane < c.N) {
          st[lane] = lg[0];
          st[c.N + lane] = rr[0];
        }
        if (lane + 32 < c.N) {
          st[lane + 32] = lg[1];
          st[c.N + lane + 32] = rr[1];
        }
        if (lane == 0) {
          st[2 * c.N] = m;
          st[2 * c.N + 1] = m + logf(l);
        }
      }
      __syncwarp();

      // ---- phase B: weighted sum of the raw rows ----
#pragma unroll
      for (int cc = 0; cc < CPT; ++cc) {
        const int chunk = tig + cc * c.tg;
        if (chunk < c.row_chunks) {
          float o[VEC];
#pragma unroll
          for (int e = 0; e < VEC; ++e) o[e] = 0.f;
          for (int n = 0; n < c.N; ++n) {
            const float al = alpha[n];
            float x[VEC];
            Dt<T>::unpack(lds128(tile + (size_t)n * c.row_bytes + chunk * 16), x);
#pragma unroll
            for (int e = 0; e < VEC; ++e) o[e] = fmaf(al, x[e], o[e]);
          }
          stg128(orow + chunk * VEC, Dt<T>::pack(o));
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
}

template <typename T, bool SOL>
static cudaError_t launch_fwd_t(const TileCfg& c, int grid, int cpt, const void* v, const void* w,
                                int w_dtype, void* out, float* stats, cudaStream_t st) {
  const size_t smem = tile_smem_layout(c).total;
  const dim3 block(32 + c.groups * c.tg);
  const T* vp = static_cast<const T*>(v);
  T* op = static_cast<T*>(out);
  switch (cpt) {
    case 1:
      return launch_smem(tile_fwd_kernel<T, 1, SOL>, grid, block, smem, st, vp, w, w_dtype, op,
                         stats, c);
    case 2:
      return launch_smem(tile_fwd_kernel<T, 2, SOL>, grid, block, smem, st, vp, w, w_dtype, op,
                         stats, c);
    case 4:
      return launch_smem(tile_fwd_kernel<T, 4, SOL>, grid, block, smem, st, vp, w, w_dtype, op,
                         stats, c);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_tile_fwd(const TileCfg& c, int grid, int cpt, int dtype, const void* v,
                            const void* w, int w_dtype, void* out, float* stats, cudaStream_t st) {
  switch (dtype) {
    case SY_BF16:
      return launch_fwd_t<__nv_bfloat16, false>(c, grid, cpt, v, w, w_dtype, out, stats, st);
    case SY_F16:
      return launch_fwd_t<__half, false>(c, grid, cpt, v, w, w_dtype, out, stats, st);
    case SY_F32:
      return launch_fwd_t<float, false>(c, grid, cpt, v, w, w_dtype, out, stats, st);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_tile_sol(const TileCfg& c, int grid, int cpt, int dtype, const void* v,
                            void* out, cudaStream_t st) {
  switch (dtype) {
    case SY_BF16:
      return launch_fwd_t<__nv_bfloat16, true>(c, grid, cpt, v, nullptr, SY_F32, out, nullptr, st);
    case SY_F16:
      return launch_fwd_t<__half, true>(c, grid, cpt, v, nullptr, SY_F32, out, nullptr, st);
    case SY_F32:
      return launch_fwd_t<float, true>(c, grid, cpt, v, nullptr, SY_F32, out, nullptr, st);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace sy
