// sy_exchange.cu -- the cross-GPU dw sum of token-sharded training, fused with
// the fixed-order reduction of the backward's partial rows.
//
// With the token axis split across ranks, every rank's backward leaves P fp32
// partial rows of length L (L = D for the single-query operator, S*D for the
// batched one); the full-batch gradient is the sum over all ranks of the sum
// of their rows. Each rank owns a buffer that every peer can address (NVLink
// peer mappings, set up by the host) holding two fp32 slots of L floats and
// world * nblk uint32 flags, nblk = ceil(L / 32): one flag per (source rank,
// 32-column block). One launch per rank, as a programmatic dependent of the
// backward, does for every 32-column block b:
//
//   1. sum the P partial rows of the block's columns in the fixed order of
//      sy_dw_reduce (8 warps, warp w taking rows w, w+8, ..., then the 8 warp
//      sums in warp order), so the rank's own row is bitwise sy_dw_reduce's;
//   2. store it into the rank's own slot `tag & 1`, then announce: store `tag`
//      into flag[rank][b] of every rank (system-scope release store);
//   3. wait until this rank's flags [r][b] hold `tag` for every rank r
//      (acquire loads, bounded by `wait_limit_ns`: on timeout the block's
//      output is NaN, the device error word gets kDevErrWaitTimeout and the
//      optional fail word gets the tag -- nothing hangs);
//   4. add the ranks' slot columns in rank order 0..world-1 (the own one from
//      registers, the others with plain peer loads) and write the result in
//      the output dtype: bitwise the same on every rank, and bitwise the sum an
//      all-gather of the ranks' sy_dw_reduce rows followed by a rank-order fp32
//      sum gives.
//
// Every block only waits on the same block of its peers, and the grid is
// small enough to be resident at once (a grid-stride loop covers larger L),
// so no CTA waits on a CTA of its own GPU that has not been scheduled.
//
// Slots alternate by tag parity: a rank rewrites a slot two calls later, and by
// then every peer has announced the next tag for that block, which it only does
// after its whole previous call -- reads of this slot included -- finished
// (stream order). Tags increase by one per call and compare modulo 2^32.
//
// Compared with a separate reduction kernel followed by an exchange kernel, the
// fusion removes one launch and one kernel boundary from the end of every
// sharded backward, and lets each block's exchange start as soon as its own
// columns are summed.
#include <cstdint>

#include "sy_common.cuh"

namespace sy {
namespace {

constexpr int kExThreads = 256;  // 8 warps: the partial-row sum of sy_dw_reduce
constexpr int kExMaxWorld = 64;
constexpr unsigned long long kExDefaultWaitNs = kWaitLimitNs;

// The announcement: a system-scope release store per destination rank, after
// the warp's slot stores. __syncwarp orders the other lanes' slot stores
// before the announcing lane's release, and a release is cumulative, so a peer
// that acquires the flag also sees every lane's slot value. 0 (shipped): the
// release store alone; 1: an explicit __threadfence_system() before it as
// well; 2: fence.acq_rel.sys before it. Measured on two B200s (per-phase
// device counters): the explicit fence adds ~3.5 us to the announcement and
// to the step, with no effect on the results.
#ifndef SY_TUNE_EXCHANGE_FENCE
#define SY_TUNE_EXCHANGE_FENCE 0
#endif

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Peer slots are re-read every second call at the same address: never serve
// them from a cache line filled by an earlier call.
__device__ __forceinline__ float ld_volatile_f(const float* p) {
  float v;
  asm volatile("ld.volatile.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kExThreads)
    reduce_exchange_kernel(const float* __restrict__ part, long long P, long long L,
                           const unsigned long long* __restrict__ bases, int world, int rank,
                           long long slot_off, long long flag_off, unsigned tag,
                           void* __restrict__ out, int out_dtype, unsigned long long limit_ns,
                           unsigned long long* __restrict__ timing,
                           unsigned* __restrict__ fail_word) {
  __shared__ float slice[8][33];
  // Everything below reads the backward's partial rows.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const unsigned long long t_entry = globaltimer_ns();
  const int lane = threadIdx.x & 31;
  const int wp = threadIdx.x >> 5;
  const long long nblk = (L + 31) / 32;
  const unsigned long long own = bases[rank];
  unsigned* const own_flags = reinterpret_cast<unsigned*>(own + flag_off);
  float* const own_slot = reinterpret_cast<float*>(own + slot_off);

  bool failed = false;  // warp 0: a wait of this CTA ran out; later blocks fail at once
  for (long long blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
    const long long col = blk * 32 + lane;
    // 1. this rank's sum of its partial rows (sy_dw_reduce's order)
    const float acc = col < L ? partial_rows_warp_sum(part, P, L, col, wp) : 0.f;
    slice[wp][lane] = acc;
    __syncthreads();
    if (wp == 0) {
      const unsigned long long t_reduced = lane == 0 ? globaltimer_ns() : 0ull;
      float mine = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) mine += slice[i][lane];
      // 2. own slot, then the announcement to every rank
      if (col < L) own_slot[col] = mine;
      __syncwarp();
      unsigned long long t_announced = 0;
      for (int r = lane; r < world; r += 32) {
#if SY_TUNE_EXCHANGE_FENCE == 1
        __threadfence_system();
#elif SY_TUNE_EXCHANGE_FENCE == 2
        asm volatile("fence.acq_rel.sys;" ::: "memory");
#endif
        st_release_sys(reinterpret_cast<unsigned*>(bases[r] + flag_off) + (long long)rank * nblk + blk,
                       tag);
      }
      if (lane == 0) t_announced = globaltimer_ns();
      // 3. bounded wait for every rank's announcement of this block
      bool ok = !failed;
      for (int r = lane; ok && r < world; r += 32) {
        const unsigned* f = own_flags + (long long)r * nblk + blk;
        const unsigned long long t0 = globaltimer_ns();
        for (uint32_t it = 0; (int)(ld_acquire_sys(f) - tag) < 0; ++it) {
          if ((it & 63u) == 63u && globaltimer_ns() - t0 > limit_ns) {
            ok = false;
            break;
          }
        }
      }
      ok = __all_sync(0xffffffffu, ok);
      failed = !ok;
      const unsigned long long t_seen = lane == 0 ? globaltimer_ns() : 0ull;
      // 4. rank-order sum (or the poison value after a timeout)
      if (col < L) {
        float total;
        if (ok) {
          total = rank == 0 ? mine : ld_volatile_f(reinterpret_cast<const float*>(bases[0] + slot_off) + col);
          for (int r = 1; r < world; ++r)
            total += r == rank ? mine
                               : ld_volatile_f(reinterpret_cast<const float*>(bases[r] + slot_off) + col);
        } else {
          total = __int_as_float(0x7fc00000);  // quiet NaN: the gradient is unusable
        }
        store_any(out, out_dtype, col, total);
      }
      if (!ok && lane == 0) {
        record_device_error(kDevErrWaitTimeout);
        if (fail_word) *reinterpret_cast<volatile unsigned*>(fail_word) = tag;
      }
      // timing[8] (block 0 of the call): calls; total and largest time from
      // the announcement to the last peer's flag; total time from the
      // kernel's start (after the backward completed) to the end of the
      // block's sum; and the totals of its phases: the partial-row sum, the
      // slot store and announcement, the peer reads and the output store
      if (timing && lane == 0 && blk == 0) {
        const unsigned long long t_end = globaltimer_ns();
        const unsigned long long wait = t_seen - t_announced;
        atomicAdd(timing + 0, 1ull);
        atomicAdd(timing + 1, wait);
        atomicMax(timing + 2, wait);
        atomicAdd(timing + 3, t_end - t_entry);
        atomicAdd(timing + 4, t_reduced - t_entry);
        atomicAdd(timing + 5, t_announced - t_reduced);
        atomicAdd(timing + 6, t_end - t_seen);
      }
    }
    __syncthreads();  // slice is reused by the next block of this CTA
  }
}

int esize(int dtype) { return dtype == SY_F32 ? 4 : ((dtype == SY_BF16 || dtype == SY_F16) ? 2 : 0); }

}  // namespace
}  // namespace sy

extern "C" int64_t sy_dw_exchange_flags(int64_t L, int world) {
  if (L < 0 || world < 1 || world > sy::kExMaxWorld) return -SY_ERR_ARG;
  return (int64_t)world * ((L + 31) / 32);
}

extern "C" int sy_dw_exchange(const float* dw_partial, int64_t P, int64_t L, const void* peer_bases,
                              int world, int rank, int64_t slot_off, int64_t flag_off, uint32_t tag,
                              void* dw, int dw_dtype, uint64_t wait_limit_ns,
                              unsigned long long* timing, unsigned int* fail_word,
                              sy_stream_t stream) {
  using namespace sy;
  if (!esize(dw_dtype)) return SY_ERR_DTYPE;
  if (world < 1 || world > kExMaxWorld || rank < 0 || rank >= world || L < 0 || P < 1)
    return SY_ERR_ARG;
  if (slot_off < 0 || flag_off < 0 || (slot_off % 4) != 0 || (flag_off % 4) != 0) return SY_ERR_ARG;
  if (L == 0) return SY_OK;
  if (!dw_partial || !peer_bases || !dw) return SY_ERR_ARG;
  if (timing && (reinterpret_cast<uintptr_t>(timing) & 7u)) return SY_ERR_ARG;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return SY_ERR_CUDA;
  const long long nblk = (L + 31) / 32;
  long long grid = nblk < 2LL * sms ? nblk : 2LL * sms;  // resident at once (small CTAs)
  if (grid < 1) grid = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kExThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, reduce_exchange_kernel, dw_partial, (long long)P, (long long)L,
                         static_cast<const unsigned long long*>(peer_bases), world, rank,
                         (long long)slot_off, (long long)flag_off, (unsigned)tag, dw, dw_dtype,
                         (unsigned long long)(wait_limit_ns ? wait_limit_ns : kExDefaultWaitNs),
                         timing, fail_word);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? SY_OK : SY_ERR_CUDA;
}
