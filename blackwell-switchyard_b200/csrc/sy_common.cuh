// sy_common.cuh -- device building blocks shared by every switchyard kernel.
//
// * dtype traits: one 16-byte "chunk" of a row (8 bf16/f16 or 4 fp32) is the
//   unit every fast kernel loads, converts to fp32, and stores.
// * mbarrier + cp.async.bulk wrappers (sm_90+ PTX, used here on sm_100a) with
//   bounded waits that record a device error word instead of hanging.
// * a warp "reduce-scatter" that sums 16 per-lane values across the warp in 15
//   shuffles, leaving value i's warp total in lanes 2i and 2i+1.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/switchyard_b200.h"

namespace sy {

// ---------------------------------------------------------------------------
// Device error word. Bit flags; read and cleared by sy_device_error().
// ---------------------------------------------------------------------------
enum : unsigned { kDevErrWaitTimeout = 1u, kDevErrBadPlan = 2u };
extern __device__ unsigned int g_device_error;

// A legitimate wait in these kernels lasts microseconds (one HBM round trip
// plus a few tiles of compute). Two seconds means something is broken.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_device_error(unsigned flag) {
  atomicOr(&g_device_error, flag);
}

// Warp `wp`'s share (of 8 warps) of the fixed-order sum of the fp32 partial
// rows part[P, L] at column `col`: rows wp, wp + 8, wp + 16, ... added in
// increasing order, 32 loads in flight per batch. The dw reduction adds the 8
// warp shares in warp order after it; every kernel that reduces partial rows
// uses this so their results agree bitwise.
__device__ __forceinline__ float partial_rows_warp_sum(const float* __restrict__ part, long long P,
                                                       long long L, long long col, int wp) {
  float acc = 0.f;
  for (long long p0 = wp; p0 < P; p0 += 8 * 32) {
    float x[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const long long p = p0 + 8 * i;
      x[i] = p < P ? __ldcs(part + p * L + col) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) acc += x[i];
  }
  return acc;
}

// ---------------------------------------------------------------------------
// dtype traits
// ---------------------------------------------------------------------------
template <typename T>
struct Dt;

template <>
struct Dt<__nv_bfloat16> {
  static constexpr int kVec = 8;  // elements per 16-byte chunk
  static constexpr int kCode = SY_BF16;
  __device__ __forceinline__ static void unpack(const uint4& u, float* x) {
    // bf16 -> fp32 is exact: the bf16 bits are the high half of the fp32.
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[2 * i] = __uint_as_float(w[i] << 16);
      x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  __device__ __forceinline__ static uint4 pack(const float* x) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
  __device__ __forceinline__ static float to_f(__nv_bfloat16 h) { return __bfloat162float(h); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float f) { return __float2bfloat16_rn(f); }
};

template <>
struct Dt<__half> {
  static constexpr int kVec = 8;
  static constexpr int kCode = SY_F16;
  __device__ __forceinline__ static void unpack(const uint4& u, float* x) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 f = __half22float2(h);
      x[2 * i] = f.x;
      x[2 * i + 1] = f.y;
    }
  }
  __device__ __forceinline__ static uint4 pack(const float* x) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
  __device__ __forceinline__ static float to_f(__half h) { return __half2float(h); }
  __device__ __forceinline__ static __half from_f(float f) { return __float2half_rn(f); }
};

template <>
struct Dt<float> {
  static constexpr int kVec = 4;
  static constexpr int kCode = SY_F32;
  __device__ __forceinline__ static void unpack(const uint4& u, float* x) {
    x[0] = __uint_as_float(u.x);
    x[1] = __uint_as_float(u.y);
    x[2] = __uint_as_float(u.z);
    x[3] = __uint_as_float(u.w);
  }
  __device__ __forceinline__ static uint4 pack(const float* x) {
    return make_uint4(__float_as_uint(x[0]), __float_as_uint(x[1]), __float_as_uint(x[2]),
                      __float_as_uint(x[3]));
  }
  __device__ __forceinline__ static float to_f(float h) { return h; }
  __device__ __forceinline__ static float from_f(float f) { return f; }
};

// Load element i of a vector whose dtype is only known at run time (used for
// the query w, which the reference accepts in any floating dtype).
__device__ __forceinline__ float load_any(const void* p, int dtype, long long i) {
  if (dtype == SY_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == SY_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_any(void* p, int dtype, long long i, float x) {
  if (dtype == SY_BF16)
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
  else if (dtype == SY_F16)
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(x);
  else
    reinterpret_cast<float*>(p)[i] = x;
}

// ---------------------------------------------------------------------------
// shared-memory / global vector access
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 lds128(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}

// A shared-memory float4 load the compiler may not merge with another.
__device__ __forceinline__ float4 lds128_f4_volatile(const void* p) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
  return v;
}

__device__ __forceinline__ void stg128(void* p, const uint4& v) {
  // Output is written once and not re-read by this kernel: stream it.
  __stcs(reinterpret_cast<uint4*>(p), v);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier + bulk async copy (PTX ISA 8.x, sm_90+)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Suspend-time hint of the waits, in ns (0: none). With a hint a waiting
// thread sleeps until the phase completes or the hint elapses, instead of
// returning at once and spinning (issue slots the working warps need).
#ifndef SY_TUNE_WAIT_HINT_NS
#define SY_TUNE_WAIT_HINT_NS 0
#endif

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
#if SY_TUNE_WAIT_HINT_NS > 0
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "n"(SY_TUNE_WAIT_HINT_NS)
      : "memory");
#else
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
#endif
  return ok != 0;
}

// Wait for the phase with the given parity to complete. Bounded: after
// kWaitLimitNs it records kDevErrWaitTimeout and returns false; the caller
// then stops issuing work and returns. (With a suspend hint every attempt can
// sleep, so the clock is read after every failed attempt.)
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(a, parity)) return true;
    if ((SY_TUNE_WAIT_HINT_NS > 0 || (it & 255u) == 0) && globaltimer_ns() - t0 > kWaitLimitNs) {
      record_device_error(kDevErrWaitTimeout);
      return false;
    }
  }
}

#ifndef SY_TUNE_L2HINT
#define SY_TUNE_L2HINT 1
#endif

// Global -> shared bulk copy (no tensor map; both addresses 16-byte aligned,
// size a multiple of 16). Completion is signalled as transaction bytes on
// `bar`. The L2 policy marks the source evict-first: every byte of v is read
// exactly once per call.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
#if SY_TUNE_L2HINT
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
#else
  (void)policy;
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
#endif
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Programmatic dependent launch. pdl_trigger: the next kernel on the stream
// (if launched as a programmatic dependent) may launch once every CTA of this
// one has triggered or exited. pdl_wait: block until the previous kernel on
// the stream has completed and its writes are visible (a no-op when this
// kernel was launched normally); called before a kernel's first global read.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Order this thread's (and, through a preceding barrier, its group's)
// generic-proxy reads of shared memory before async-proxy (bulk copy) writes
// to the same bytes.
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Named barrier over `nthreads` threads (a multiple of 32). id 0 is
// __syncthreads; the kernels use 1..15.
__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------
// packed fp32 helpers (float2 = one fma.rn.f32x2 lane pair)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

// Unpack one 16-byte chunk into VEC/2 float2 pairs (elements 2i, 2i+1).
template <typename T>
__device__ __forceinline__ void unpack2(const uint4& u, float2* p) {
  float x[Dt<T>::kVec];
  Dt<T>::unpack(u, x);
#pragma unroll
  for (int i = 0; i < Dt<T>::kVec / 2; ++i) p[i] = make_float2(x[2 * i], x[2 * i + 1]);
}

// Mixed-precision FMA on packed 16-bit pairs (sm_100: fma.rn.f32.{bf16,f16}):
// acc.x += lo(a) * lo(b), acc.y += hi(a) * hi(b), one fp32 rounding each. The
// 16-bit operands convert to fp32 exactly and their product is exact in fp32,
// so this equals __ffma2_rn on the unpacked values -- without the unpacking.
template <typename T>
__device__ __forceinline__ void mixfma2(float2& acc, uint32_t a, uint32_t b);
template <>
__device__ __forceinline__ void mixfma2<__nv_bfloat16>(float2& acc, uint32_t a, uint32_t b) {
  asm("{\n\t.reg .b16 al, ah, bl, bh;\n\tmov.b32 {al, ah}, %2;\n\tmov.b32 {bl, bh}, %3;\n\t"
      "fma.rn.f32.bf16 %0, al, bl, %0;\n\tfma.rn.f32.bf16 %1, ah, bh, %1;\n\t}"
      : "+f"(acc.x), "+f"(acc.y)
      : "r"(a), "r"(b));
}
template <>
__device__ __forceinline__ void mixfma2<__half>(float2& acc, uint32_t a, uint32_t b) {
  asm("{\n\t.reg .b16 al, ah, bl, bh;\n\tmov.b32 {al, ah}, %2;\n\tmov.b32 {bl, bh}, %3;\n\t"
      "fma.rn.f32.f16 %0, al, bl, %0;\n\tfma.rn.f32.f16 %1, ah, bh, %1;\n\t}"
      : "+f"(acc.x), "+f"(acc.y)
      : "r"(a), "r"(b));
}

template <typename T>
__device__ __forceinline__ uint4 pack2(const float2* p) {
  float x[Dt<T>::kVec];
#pragma unroll
  for (int i = 0; i < Dt<T>::kVec / 2; ++i) {
    x[2 * i] = p[i].x;
    x[2 * i + 1] = p[i].y;
  }
  return Dt<T>::pack(x);
}

// ---------------------------------------------------------------------------
// warp reductions
// ---------------------------------------------------------------------------
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(kFull, x, o);
  return x;
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(kFull, x, o));
  return x;
}

// Sum each of 16 per-lane values over the 32 lanes of the warp.
// Step k (offset 16, 8, 4, 2) halves the live set: the lane whose offset bit
// is set keeps the upper half and sends the lower half to its partner, which
// keeps the lower half. After four steps lane L holds the sum over 16 lanes of
// value (L >> 1); the final xor-1 step completes it, so lanes 2i and 2i+1
// both hold the warp total of value i (bitwise equal: a+b == b+a).
// 8 + 4 + 2 + 1 + 1 = 16 shuffles instead of 16 * 5 = 80 for separate sums.
// The summation order is fixed, so results are deterministic.
__device__ __forceinline__ float warp_reduce_scatter16(float (&a)[16], int lane) {
  {
    const bool up = lane & 16;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float send = up ? a[i] : a[i + 8];
      const float keep = up ? a[i + 8] : a[i];
      a[i] = keep + __shfl_xor_sync(kFull, send, 16);
    }
  }
  {
    const bool up = lane & 8;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float send = up ? a[i] : a[i + 4];
      const float keep = up ? a[i + 4] : a[i];
      a[i] = keep + __shfl_xor_sync(kFull, send, 8);
    }
  }
  {
    const bool up = lane & 4;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float send = up ? a[i] : a[i + 2];
      const float keep = up ? a[i + 2] : a[i];
      a[i] = keep + __shfl_xor_sync(kFull, send, 4);
    }
  }
  {
    const bool up = lane & 2;
    const float send = up ? a[0] : a[1];
    const float keep = up ? a[1] : a[0];
    a[0] = keep + __shfl_xor_sync(kFull, send, 2);
  }
  return a[0] + __shfl_xor_sync(kFull, a[0], 1);
}

}  // namespace sy
