// sy_exchange.cu -- the cross-GPU dw sum of token-sharded training, fused with
// the fixed-order reduction of the backward's partial rows.
//
// With the token axis split across ranks, every rank's backward leaves P fp32
// partial rows of length L (L = D for the single-query operator, S*D for the
// batched one); the full-batch gradient is the sum over all ranks of the sum
// of their rows. Each rank owns a buffer that every peer can address (NVLink
// peer mappings, set up by the host): two slots, each holding one 8-byte word
// per (source rank, column). A word is the fp32 value in its low half and the
// call's 32-bit tag in its high half. One launch per rank, as a programmatic
// dependent of the backward, does for every 32-column block:
//
//   1. sum the P partial rows of the block's columns in the fixed order of
//      sy_dw_reduce (8 warps, warp w taking rows w, w+8, ..., then the 8 warp
//      sums in warp order), so the rank's own row is bitwise sy_dw_reduce's;
//   2. push: every lane stores its column's word (value, tag) into slot
//      `tag & 1`, row `rank`, of every other rank's buffer -- one 8-byte
//      relaxed system-scope store per peer, fire and forget;
//   3. add the ranks' values in rank order 0..world-1: its own from registers,
//      each peer's by polling the word in its OWN buffer (local memory) until
//      the word's tag is this call's (bounded by `wait_limit_ns`: on timeout
//      the block's output is NaN, the device error word gets
//      kDevErrWaitTimeout and the optional fail word gets the tag -- nothing
//      hangs); the result is written in the output dtype: bitwise the same on
//      every rank, and bitwise the sum an all-gather of the ranks'
//      sy_dw_reduce rows followed by a rank-order fp32 sum gives.
//
// The value and its tag travel in one naturally aligned 8-byte store, which is
// single-copy atomic: a reader sees either the old word or the whole new one,
// so no fence orders data before a flag and no reader crosses NVLink (the
// flag-in-data scheme of low-latency collective protocols). A first version
// stored the value in the rank's own slot, announced it with a system-scope
// release store of a separate flag and let peers read the slot remotely; on
// two B200s the release cost 2-4 us and the remote read ~2 us per step.
//
// Every block only waits on the same columns of its peers, and the grid is
// small enough to be resident at once (a grid-stride loop covers larger L), so
// no CTA waits on a CTA of its own GPU that has not been scheduled.
//
// Slots alternate by tag parity: a rank writes a peer's slot again two calls
// later, and it only starts that call after it received the peer's words of
// the call in between, which the peer pushes only after its own previous call
// -- reads of that slot included -- finished (stream order). Tags increase by
// one per call (never 0: the buffer starts zeroed) and compare modulo 2^32.
#include <cstdint>

#include "sy_common.cuh"

namespace sy {
namespace {

constexpr int kExThreads = 256;  // 8 warps: the partial-row sum of sy_dw_reduce
constexpr int kExMaxWorld = 64;
constexpr unsigned long long kExDefaultWaitNs = kWaitLimitNs;

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kExThreads)
    reduce_exchange_kernel(const float* __restrict__ part, long long P, long long L,
                           const unsigned long long* __restrict__ bases, int world, int rank,
                           long long buf_off, unsigned tag, void* __restrict__ out, int out_dtype,
                           unsigned long long limit_ns, unsigned long long* __restrict__ timing,
                           unsigned* __restrict__ fail_word) {
  __shared__ float slice[8][33];
  // Everything below reads the backward's partial rows.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const unsigned long long t_entry = globaltimer_ns();
  const int lane = threadIdx.x & 31;
  const int wp = threadIdx.x >> 5;
  const long long nblk = (L + 31) / 32;
  // word (slot, src, col) of a rank's buffer
  const long long slot_words = (long long)(tag & 1u) * world * L;
  auto word_at = [&](unsigned long long base, int src, long long col) {
    return reinterpret_cast<unsigned long long*>(base + buf_off) + slot_words + (long long)src * L + col;
  };
  const unsigned long long own = bases[rank];

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
      // 2. push (value, tag) to every other rank
      const unsigned long long word =
          ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(mine);
      if (col < L)
        for (int r = 0; r < world; ++r)
          if (r != rank) st_relaxed_sys_u64(word_at(bases[r], rank, col), word);
      const unsigned long long t_announced = lane == 0 ? globaltimer_ns() : 0ull;
      // 3. rank-order sum, each peer's word polled in this rank's own buffer
      bool ok = !failed;
      float total = 0.f;
      if (col < L) {
        for (int r = 0; r < world && ok; ++r) {
          float x = mine;
          if (r != rank) {
            const unsigned long long* wq = word_at(own, r, col);
            unsigned long long got = ld_relaxed_sys_u64(wq);
            const unsigned long long t0 = globaltimer_ns();
            for (uint32_t it = 0; (unsigned)(got >> 32) != tag; ++it) {
              if ((it & 63u) == 63u && globaltimer_ns() - t0 > limit_ns) {
                ok = false;
                break;
              }
              got = ld_relaxed_sys_u64(wq);
            }
            x = __uint_as_float((unsigned)got);
          }
          total = r == 0 ? x : total + x;
        }
      }
      ok = __all_sync(0xffffffffu, ok);
      failed = !ok;
      const unsigned long long t_seen = lane == 0 ? globaltimer_ns() : 0ull;
      if (col < L) store_any(out, out_dtype, col, ok ? total : __int_as_float(0x7fc00000));
      if (!ok && lane == 0) {
        record_device_error(kDevErrWaitTimeout);
        if (fail_word) *reinterpret_cast<volatile unsigned*>(fail_word) = tag;
      }
      // timing[8] (block 0 of the call): calls; total and largest time from
      // the push to the last peer word; total time from the kernel's start
      // (after the backward completed) to the end of the block's sum; and the
      // totals of its phases: the partial-row sum, the pushes, the wait with
      // the rank-order sum and the output store
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

extern "C" int64_t sy_dw_exchange_bytes(int64_t L, int world) {
  if (L < 0 || world < 1 || world > sy::kExMaxWorld) return -SY_ERR_ARG;
  return (int64_t)2 * world * L * 8;
}

extern "C" int sy_dw_exchange(const float* dw_partial, int64_t P, int64_t L, const void* peer_bases,
                              int world, int rank, int64_t buf_off, uint32_t tag, void* dw,
                              int dw_dtype, uint64_t wait_limit_ns, unsigned long long* timing,
                              unsigned int* fail_word, sy_stream_t stream) {
  using namespace sy;
  if (!esize(dw_dtype)) return SY_ERR_DTYPE;
  if (world < 1 || world > kExMaxWorld || rank < 0 || rank >= world || L < 0 || P < 1 || tag == 0)
    return SY_ERR_ARG;
  if (buf_off < 0 || (buf_off % 8) != 0) return SY_ERR_ARG;
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
                         (long long)buf_off, (unsigned)tag, dw, dw_dtype,
                         (unsigned long long)(wait_limit_ns ? wait_limit_ns : kExDefaultWaitNs),
                         timing, fail_word);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? SY_OK : SY_ERR_CUDA;
}
