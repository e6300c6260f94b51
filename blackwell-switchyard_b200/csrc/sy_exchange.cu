// sy_exchange.cu -- the cross-GPU dw sum of token-sharded training.
//
// With the token axis split across ranks, every rank's backward produces an
// fp32 dw over its own tokens; the full-batch dw is their sum. Each rank keeps
// two fp32 slots of D floats and an array of `world` uint32 flags in memory
// that every peer can address (NVLink peer mappings; the host side sets them up
// and passes each rank's base address). One call, on every rank, with the
// rank's own dw already written into slot `tag & 1` by an earlier kernel on the
// same stream:
//
//   1. announce: store `tag` into flag[rank] of every rank (release, system
//      scope, after a system fence), i.e. "my slot for this tag is complete";
//   2. wait until this rank's own flag array holds `tag` for every rank
//      (acquire loads, bounded by a 2 s limit that records the device error word
//      instead of hanging);
//   3. read all ranks' slots with plain peer loads and add them in rank order
//      0..world-1 (so every rank gets the bitwise-same result), writing dw in
//      the requested dtype.
//
// Slots alternate by tag parity: a rank reuses a slot two calls later, and by
// then every peer has announced the next tag, which it only does after its own
// reads of the previous one finished (stream order) -- so no slot is rewritten
// while a peer may still read it. Tags increase by one per call and are
// compared modulo 2^32.
#include <cstdint>

#include "sy_common.cuh"

namespace sy {
namespace {

constexpr int kExThreads = 256;
constexpr int kExMaxWorld = 64;

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Peer data is re-read every second call at the same address: never serve it
// from a cache line filled by an earlier call.
__device__ __forceinline__ float ld_volatile_f(const float* p) {
  float v;
  asm volatile("ld.volatile.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float4 ld_volatile_f4(const float* p) {
  float4 v;
  asm volatile("ld.volatile.global.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__global__ void __launch_bounds__(kExThreads)
    dw_exchange_kernel(const unsigned long long* __restrict__ bases, int world, int rank,
                       long long slot_off, long long flag_off, unsigned tag, long long D,
                       void* __restrict__ dw, int dw_dtype) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  // 1. announce (one thread per destination rank, first CTA only)
  if (blockIdx.x == 0 && (int)threadIdx.x < world) {
    __threadfence_system();
    unsigned* f = reinterpret_cast<unsigned*>(bases[threadIdx.x] + flag_off) + rank;
    st_release_sys(f, tag);
  }
  __syncthreads();
  // 2. every CTA waits for all ranks' announcements of this tag
  if ((int)threadIdx.x < world) {
    const unsigned* f = reinterpret_cast<const unsigned*>(bases[rank] + flag_off) + threadIdx.x;
    const unsigned long long t0 = globaltimer_ns();
    for (uint32_t it = 0; (int)(ld_acquire_sys(f) - tag) < 0; ++it) {
      if ((it & 63u) == 63u && globaltimer_ns() - t0 > kWaitLimitNs) {
        record_device_error(kDevErrWaitTimeout);
        ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  if (!ok) return;
  // 3. rank-order sum, 4 columns per thread (slots are 16-byte aligned)
  const long long stride = (long long)gridDim.x * blockDim.x * 4;
  for (long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4; i < D; i += stride) {
    if (i + 4 <= D) {
      float4 acc = ld_volatile_f4(reinterpret_cast<const float*>(bases[0] + slot_off) + i);
      for (int r = 1; r < world; ++r) {
        const float4 x = ld_volatile_f4(reinterpret_cast<const float*>(bases[r] + slot_off) + i);
        acc.x += x.x;
        acc.y += x.y;
        acc.z += x.z;
        acc.w += x.w;
      }
      store_any(dw, dw_dtype, i, acc.x);
      store_any(dw, dw_dtype, i + 1, acc.y);
      store_any(dw, dw_dtype, i + 2, acc.z);
      store_any(dw, dw_dtype, i + 3, acc.w);
    } else {
      for (long long k = i; k < D; ++k) {
        float acc = ld_volatile_f(reinterpret_cast<const float*>(bases[0] + slot_off) + k);
        for (int r = 1; r < world; ++r)
          acc += ld_volatile_f(reinterpret_cast<const float*>(bases[r] + slot_off) + k);
        store_any(dw, dw_dtype, k, acc);
      }
    }
  }
}

int esize(int dtype) { return dtype == SY_F32 ? 4 : ((dtype == SY_BF16 || dtype == SY_F16) ? 2 : 0); }

}  // namespace
}  // namespace sy

extern "C" int sy_dw_exchange(const void* peer_bases, int world, int rank, int64_t slot_off,
                              int64_t flag_off, uint32_t tag, int64_t D, void* dw, int dw_dtype,
                              sy_stream_t stream) {
  using namespace sy;
  if (!esize(dw_dtype)) return SY_ERR_DTYPE;
  if (world < 1 || world > kExMaxWorld || rank < 0 || rank >= world || D < 0) return SY_ERR_ARG;
  if (slot_off < 0 || flag_off < 0 || (slot_off % 16) != 0 || (flag_off % 4) != 0)
    return SY_ERR_ARG;
  if (D == 0) return SY_OK;
  if (!peer_bases || !dw) return SY_ERR_ARG;
  const long long per_cta = (long long)kExThreads * 4;
  long long grid = (D + per_cta - 1) / per_cta;
  if (grid > 1024) grid = 1024;
  dw_exchange_kernel<<<(unsigned)grid, kExThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const unsigned long long*>(peer_bases), world, rank, (long long)slot_off,
      (long long)flag_off, tag, (long long)D, dw, dw_dtype);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SY_OK : SY_ERR_CUDA;
}
