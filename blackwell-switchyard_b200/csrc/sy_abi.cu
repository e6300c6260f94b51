// sy_abi.cu -- the extern "C" entry points declared in include/switchyard_b200.h:
// argument validation, kernel planning and dispatch. No device allocation
// happens anywhere in this library.
#include <climits>
#include <cstdio>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "sy_batched.cuh"
#include "sy_reg.cuh"
#include "sy_stream.cuh"
#include "sy_stream_batched.cuh"
#include "sy_stream_bwd.cuh"
#include "sy_tile.cuh"

// Planner tuning knobs. The defaults are the shipped configuration; builds
// with other values exist only for tuning sweeps.
#ifndef SY_TUNE_MAX_STAGES
#define SY_TUNE_MAX_STAGES 32
#endif
#ifndef SY_TUNE_GROUPS
#define SY_TUNE_GROUPS 0  // 0: as many groups as fit 256 consumer threads
#endif
#ifndef SY_TUNE_CTAS_PER_SM
#define SY_TUNE_CTAS_PER_SM 1
#endif
#ifndef SY_TUNE_PDL
#define SY_TUNE_PDL 1  // launch the dw reduction as a programmatic dependent
#endif
#ifndef SY_TUNE_STREAM_REREAD
#define SY_TUNE_STREAM_REREAD 1  // forward, 8 chunks per lane: re-read row stream first
#endif
#ifndef SY_TUNE_STREAM_BWD
#define SY_TUNE_STREAM_BWD 1  // backward: row stream before the shared-memory tile
#endif
#ifndef SY_TUNE_REREAD_CPL4
#define SY_TUNE_REREAD_CPL4 1  // forward, 2 KiB rows: re-read row stream (4 chunks per lane)
#endif
#ifndef SY_TUNE_BATCHED_REG
#define SY_TUNE_BATCHED_REG 1  // batched: the register tile where it fits (else row stream)
#endif
#ifndef SY_TUNE_BWD_L2_PCT
#define SY_TUNE_BWD_L2_PCT 0  // row-stream backward: fit rows in flight in this % of L2 (0: off)
#endif

namespace sy {

__device__ unsigned int g_device_error = 0;

namespace {

constexpr int64_t kMaxD = 1 << 24;  // D is converted to float exactly below 2^24
constexpr int kMaxDevices = 64;

struct DevInfo {
  int sms = 0;
  int max_smem = 0;  // opt-in dynamic shared memory per block
  int64_t l2 = 0;    // L2 bytes
};

// L2 assumed by sy_plan_info when it is given a device's SM count and shared
// memory instead of querying one (B200: 126 MiB).
constexpr int64_t kAssumedL2Bytes = int64_t(126) << 20;

cudaError_t dev_info(DevInfo* out) {
  static std::mutex mu;
  static DevInfo cache[kMaxDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(mu);
  if (cache[dev].sms == 0) {
    DevInfo d;
    e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&d.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return e;
    int l2 = 0;
    e = cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, dev);
    if (e != cudaSuccess) return e;
    d.l2 = l2;
    cache[dev] = d;
  }
  *out = cache[dev];
  return cudaSuccess;
}

int esize_of(int dtype) {
  switch (dtype) {
    case SY_BF16:
    case SY_F16:
      return 2;
    case SY_F32:
      return 4;
    default:
      return 0;
  }
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool al8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }

int64_t stats_stride(int64_t N) { return ((2 * N + 2) + 3) / 4 * 4; }

enum TileOp { kOpFwd = 0, kOpBwd = 1, kOpSol = 2 };
enum PlanKind { kPlanGeneric = 0, kPlanRegTile = 1, kPlanSmemTile = 2, kPlanStream = 3 };

struct TilePlan {
  int kind = kPlanGeneric;
  TileCfg c{};
  int grid = 0;
  int cpt = 0;
  int64_t smem = 0;
};

int64_t round32(int64_t x) { return (x + 31) / 32 * 32; }

// Fill in stages/groups for a tile configuration whose tg, row and scratch
// sizes are set. Returns false if fewer than two stages fit.
bool size_ring(TileCfg& c, int op, int groups, const DevInfo& di, int64_t* smem_out,
               bool per_group_rings = false) {
  int64_t body = (int64_t)c.N * c.row_bytes;
  if (op == kOpBwd) body = (int64_t)(c.N + 1) * c.row_bytes + (int64_t)c.stats_stride * 4;
  const int64_t stage = (body + 127) / 128 * 128;
  if (stage > INT_MAX / 4) return false;
  c.stage_bytes = (int)stage;
  c.groups = groups;
  c.stages = 0;
  const int64_t fixed = (int64_t)tile_smem_layout(c).total;
  // Shared memory per CTA: the whole opt-in limit at one CTA per SM; with k
  // CTAs per SM, a k-th of the SM's 228 KiB minus the 1 KiB each CTA reserves.
  const int64_t budget = SY_TUNE_CTAS_PER_SM == 1
                             ? di.max_smem
                             : (int64_t)(233472 / SY_TUNE_CTAS_PER_SM) - 1024;
  int64_t stages = (budget - fixed) / (stage + 2 * (int64_t)sizeof(uint64_t));
  if (stages > SY_TUNE_MAX_STAGES) stages = SY_TUNE_MAX_STAGES;
  if (stages < 2) return false;
  // Group g consumes tokens k = g (mod G) from stage k mod S, waiting on the
  // stage's barrier with parity (k / S) & 1. That parity test is only sound if
  // the previous token of the same stage was consumed by the same group (then
  // it has certainly landed): S must be a multiple of G. Each group also gets
  // at least two stages, so one can load while it computes on the other.
  // (The register-tile kernels give every group its own ring instead, which
  // has no such constraint.)
  // With per-group rings (the register-tile kernels refill a stage as soon as
  // the group holds it in registers) one stage per group already overlaps
  // loads with compute.
  while (groups > 1 && stages < (per_group_rings ? 1 : 2) * groups) --groups;
  if (!per_group_rings) stages = stages / groups * groups;
  c.groups = groups;
  c.stages = (int)stages;
  const int64_t total = (int64_t)tile_smem_layout(c).total;
  if (total > budget) return false;
  *smem_out = total;
  return true;
}

// Choose the kernel family and configuration for a shape. Pointer alignment
// is checked by the caller (misaligned pointers take the generic kernels).
TilePlan plan_tile(int op, int64_t N, int64_t BT, int64_t D, int dtype, const DevInfo& di) {
  TilePlan p;
  const int es = esize_of(dtype);
  if (!es || N < 1 || N > kTileMaxN || D < 1 || D > kMaxD || BT < 1 || BT > INT_MAX) return p;
  if ((D * es) % 16) return p;
  const int64_t rc = D * es / 16;  // 16-byte chunks per row

  TileCfg c{};
  c.BT = BT;
  c.N = (int)N;
  c.D = (int)D;
  c.row_chunks = (int)rc;
  c.row_bytes = (int)(D * es);
  c.stats_stride = (int)stats_stride(N);
  c.red_stride = tile_red_stride((int)N);
  const int64_t slots = (int64_t)di.sms * SY_TUNE_CTAS_PER_SM;
  const int grid = (int)(BT < slots ? BT : slots);

  // 1) register tile: exact-N kernels, the packed tile (N * CPT * 4 words)
  //    held in registers; two chunks per thread up to N = 9, else one.
  if (op != kOpSol && N <= (op == kOpFwd ? kRegFwdMaxN : kRegMaxN)) {
    // Chunks per thread: the more, the fewer warps share a token, so the
    // per-warp cost of its reductions and softmax is spread over more data
    // and more tokens are in flight per SM. Forward: up to 4 (N <= 9; the tile
    // is then kept packed), backward: up to 2 (N <= 9, more live state).
    // Never so many that a warp's lanes would sit idle.
    int cpt = 0, tg = 0;
    // The stage-held forward keeps no tile in registers: four chunks for any
    // N <= 9, in groups of (at D=2048 bf16) two warps, kHoldThreads per CTA.
    // With one stage per group its groups start in lockstep (all load, then
    // all compute), which only evens out over many tokens per SM; below
    // kHoldMinTokensPerSM the register tile (stage refilled as soon as the
    // tile is in registers) is faster.
    const bool hold = op == kOpFwd && SY_TUNE_FWD_HOLD && N <= kRegFwdMaxN &&
                      BT >= (int64_t)kHoldMinTokensPerSM * di.sms;
    const int max_cpt = hold ? 4 : (N <= kRegMaxN4 && op == kOpFwd ? 4 : (N <= kRegMaxN2 ? 2 : 1));
    for (int cand = max_cpt; cand >= 1 && !cpt; cand /= 2) {
      if (cand > 1 && rc < 32 * cand) continue;  // lanes would be idle
      const int64_t t = round32((rc + cand - 1) / cand);
      if (t <= 256 && (rc + t - 1) / t <= cand) cpt = cand, tg = (int)t;
    }
    if (cpt) {
      TileCfg rcfg = c;
      rcfg.tg = tg;
      rcfg.coef_stride = op == kOpBwd ? tile_coef_stride((int)N) : 0;  // bwd: float4 per source
      rcfg.w_smem = op == kOpBwd ? 0 : 1;  // forward reads its fp32 w from shared memory
      rcfg.hold = hold ? 1 : 0;
      int groups = (hold ? kHoldThreads : reg_threads((int)N, cpt, 16 / es, op == kOpBwd)) / tg;
      if (groups > 16) groups = 16;  // named barrier ids 1..15 (1-warp groups use none)
      if (SY_TUNE_GROUPS > 0) groups = SY_TUNE_GROUPS;
      if (size_ring(rcfg, op, groups < 1 ? 1 : groups, di, &p.smem, /*per_group_rings=*/true)) {
        p.kind = kPlanRegTile;
        p.c = rcfg;
        p.cpt = cpt;
        p.grid = grid;
        return p;
      }
    }
  }

  // 2) shared-memory tile: run-time N (up to kTileMaxN), rows re-read from
  //    the stage in the weighted sum.
  int cpt = 0, tg = 0;
  const int cands[3] = {2, 1, 4};
  for (int cand : cands) {
    const int64_t t = round32((rc + cand - 1) / cand);
    if (t <= kConsumerThreads && (rc + t - 1) / t <= cand) {
      cpt = cand;
      tg = (int)t;
      break;
    }
  }
  if (!cpt) return p;
  c.tg = tg;
  c.coef_stride = tile_coef_stride((int)N);
  int groups = kConsumerThreads / tg;
  if (SY_TUNE_GROUPS > 0) groups = SY_TUNE_GROUPS;
  if (!size_ring(c, op, groups < 1 ? 1 : groups, di, &p.smem)) return p;
  p.kind = kPlanSmemTile;
  p.c = c;
  p.cpt = cpt;
  p.grid = grid;
  return p;
}

struct StreamPlan {
  bool ok = false;
  StreamCfg c{};
  int grid = 0;
  int cpl = 0;
  int64_t smem = 0;
};

// Row-stream forward (one warp per token, online softmax): rows must be a
// multiple of 16 bytes and fit 8 16-byte chunks per lane (bf16/f16 D <= 2048,
// fp32 D <= 1024); any N.
StreamPlan plan_stream(int64_t N, int64_t BT, int64_t D, int dtype, const DevInfo& di,
                       bool sol = false) {
  StreamPlan p;
  const int es = esize_of(dtype);
  if (!es || N < 1 || D < 1 || D > kMaxD || BT < 1 || BT > INT_MAX) return p;
  if ((D * es) % 16) return p;
  const int64_t rc = D * es / 16;
  // Rows of exactly 2, 4 or 8 times 4 KiB: the split re-read kernel, K warps
  // per token. Otherwise one warp per token, rows of at most 8 chunks per lane.
  const int kw =
      (!sol && SY_TUNE_STREAM_REREAD && (rc == 512 || rc == 1024 || rc == 2048)) ? (int)(rc / 256) : 1;
  int cpl = 1;
  while (cpl * 32 * kw < rc) cpl *= 2;
  if (cpl > 8) return p;
  StreamCfg c{};
  c.BT = BT;
  c.N = (int)N;
  c.D = (int)D;
  c.row_chunks = (int)rc;
  c.row_bytes = (int)(D * es);
  c.kw = kw;
  // 2 KiB rows: the re-read stream where the register tile's stage-held
  // forward does not apply (N > 9, or fewer than kHoldMinTokensPerSM tokens
  // per SM); that one is faster from there on (5.95 vs 4.96 TB/s at N=9
  // T=32768 D=1024 bf16).
  const bool cpl4 = cpl == 4 && kw == 1 && SY_TUNE_REREAD_CPL4 &&
                    (N > kRegFwdMaxN || BT < (int64_t)kHoldMinTokensPerSM * di.sms);
  c.reread = (SY_TUNE_STREAM_REREAD && !sol && (cpl == 8 || cpl4)) ? 1 : 0;
  c.warps = stream_threads(cpl, c.reread != 0) / 32;
  if (c.reread) {
    // Whole tokens per token stream (a warp, or K warps), as even as possible:
    // with t tokens per CTA and at most M streams, k = ceil(t / M) tokens per
    // stream and ceil(t / k) streams, so no stream has more tokens than
    // necessary (4096 tokens on 148 SMs: 14 single-warp streams x 2).
    const int64_t g0 = BT < di.sms ? BT : di.sms;
    const int64_t t = (BT + g0 - 1) / g0;
    const int64_t mw = kStreamRereadThreads / 32 / kw;
    const int64_t k = (t + mw - 1) / mw;
    c.warps = (int)((t + k - 1) / k) * kw;
    if (k * N >= (int64_t)INT_MAX) return p;  // rows per stream are counted in 32 bits
  }
  c.stats_stride = (int)stats_stride(N);
  c.ring = 0;
  const int64_t fixed = (int64_t)stream_smem_layout(c).total;
  const int64_t per_row = (int64_t)(c.warps / kw) * (c.row_bytes + 8 + (kw > 1 ? 4 : 0));
  int64_t ring = (di.max_smem - fixed - 16) / per_row;
  if (ring > 8) ring = 8;
  if (ring < 2) return p;
  c.ring = (int)ring;
  const StreamSmem lay = stream_smem_layout(c);
  p.smem = (int64_t)lay.total;
  if (p.smem > di.max_smem) return p;
  // 16-byte vector accesses and bulk copies: every region on a 16-byte boundary
  if (lay.ring_off % 16 || lay.bar_off % 16 || lay.xch_off % 16 || lay.zero_off % 16) return p;
  const int64_t need = (BT + c.warps - 1) / c.warps;  // CTAs with work for every warp
  p.grid = (int)(need < di.sms ? need : di.sms);
  if (c.reread) p.grid = (int)(BT < di.sms ? BT : di.sms);
  p.c = c;
  p.cpl = cpl;
  p.ok = true;
  return p;
}

struct StreamBwdPlan {
  bool ok = false;
  StreamBwdCfg c{};
  int grid = 0;
  int64_t smem = 0;
};

// Row-stream backward: rows of exactly 32 * CPL * K chunks (CPL = 4, 2 or 1
// chunks per lane, K = 1 .. 16 warps per token), N <= 64; it runs where the
// register tile does not (N > 16, or rows over 4 KiB). Whole tokens per token
// stream, as evenly as possible (as the forward's re-read stream). The most
// chunks per lane that divide the row: fewer warps per token, fewer barriers.
// Pass B re-reads each row, normally from L2, but the rows in flight (token
// streams x SMs x N rows) can exceed L2 at large N (N = 33, 4 KiB rows: 137 MB).
// Two ways of keeping them within L2 were measured and are slower at every
// shape tried (N = 17..64, D = 1024..8192): fewer token streams (0.67 -> 0.15-0.52
// of the copy peak at N = 33 D = 2048) and fewer chunks per lane with more warps
// per token (0.67 -> 0.53); the DRAM re-reads cost less than either.
// SY_TUNE_BWD_L2_PCT > 0 keeps the second rule for experiments.
StreamBwdPlan plan_stream_bwd(int64_t N, int64_t BT, int64_t D, int dtype, const DevInfo& di) {
  StreamBwdPlan p;
  const int es = esize_of(dtype);
  if (!SY_TUNE_STREAM_BWD || !es || N < 1 || N > kStreamBwdMaxN || D < 1 || D > kMaxD ||
      BT < 1 || BT > INT_MAX)
    return p;
  if ((D * es) % 16) return p;
  const int64_t rc = D * es / 16;
  const int64_t g0 = BT < di.sms ? BT : di.sms;
  const int64_t t = (BT + g0 - 1) / g0;  // tokens per CTA
  const int64_t budget = di.l2 > 0 ? (int64_t)SY_TUNE_BWD_L2_PCT * di.l2 / 100 : 0;
  int64_t kw = 0, streams = 0, cpl = 0;
  for (int64_t c = kStreamBwdMaxCpl; c >= 1; c /= 2) {
    if (rc % (32 * c)) continue;
    const int64_t k_w = rc / (32 * c);
    if (k_w < 1 || k_w > 16) continue;
    int64_t max_streams = kStreamBwdThreads / 32 / k_w;
    if (k_w > 1 && max_streams > 15) max_streams = 15;  // named barrier ids 1..15
    const int64_t k = (t + max_streams - 1) / max_streams;  // tokens per stream
    const int64_t s = (t + k - 1) / k;
    if (k * (2 * N + 1) >= (int64_t)INT_MAX) continue;  // stream rows are counted in 32 bits
    kw = k_w, streams = s, cpl = c;
    if (budget == 0 || s * di.sms * N * (D * es) <= budget) break;
  }
  if (!cpl) return p;
  StreamBwdCfg c{};
  c.BT = BT;
  c.N = (int)N;
  c.D = (int)D;
  c.row_chunks = (int)rc;
  c.cpl = (int)cpl;
  c.row_bytes = (int)(D * es);
  c.kw = (int)kw;
  c.warps = (int)(streams * kw);
  c.stats_stride = (int)stats_stride(N);
  c.ring = 0;
  const int64_t fixed = (int64_t)stream_bwd_smem_layout(c).total;
  const int64_t per_row = streams * ((int64_t)c.row_bytes + 8 + 4);
  int64_t ring = (di.max_smem - fixed - 16) / per_row;
  if (ring > 8) ring = 8;
  if (ring < 2) return p;
  c.ring = (int)ring;
  p.smem = (int64_t)stream_bwd_smem_layout(c).total;
  if (p.smem > di.max_smem) return p;
  p.c = c;
  p.grid = (int)g0;
  p.ok = true;
  return p;
}

// Batched-query register tile: the fp32 tile (N * CPT * VEC floats per thread)
// must fit kBatchedTileFloats; as many chunks per thread as fit (fewer warps
// per token: less reduction work per query), groups of up to 256 threads, the
// queries' SB slots (S rounded up to 4, 8 or 16) in shared memory beside the
// ring.
TilePlan plan_batched(int64_t N, int64_t BT, int64_t D, int64_t S, int dtype, const DevInfo& di) {
  TilePlan p;
  if (!SY_TUNE_BATCHED_REG) return p;
  const int es = esize_of(dtype);
  if (!es || N < 1 || N > kRegMaxN || S < 1 || S > kBatchedMaxS || D < 1 || D > kMaxD ||
      BT < 1 || BT > INT_MAX)
    return p;
  if ((D * es) % 16) return p;
  const int vec = 16 / es;
  const int64_t rc = D * es / 16;
  int cpt = 0, tg = 0;
  for (int cand = 4; cand >= 1 && !cpt; cand /= 2) {
    if (N * cand * vec > kBatchedTileFloats) continue;
    if (cand > 1 && rc < 32 * cand) continue;  // lanes would be idle
    const int64_t t = round32((rc + cand - 1) / cand);
    if (t <= kBatchedThreads && (rc + t - 1) / t <= cand) cpt = cand, tg = (int)t;
  }
  if (!cpt) return p;
  TileCfg c{};
  c.BT = BT;
  c.N = (int)N;
  c.D = (int)D;
  c.row_chunks = (int)rc;
  c.row_bytes = (int)(D * es);
  c.stats_stride = (int)stats_stride(N);
  c.red_stride = batched_red_stride((int)N, (int)S);    // the blocks' warp totals
  c.coef_stride = batched_coef_stride((int)N, (int)S);  // alpha pairs of every query slot
  c.tg = tg;
  DevInfo room = di;  // the query slots take SB rows of shared memory
  room.max_smem = di.max_smem - (int)(batched_slots((int)S) * c.row_bytes) - 128;
  int64_t smem = 0;
  if (room.max_smem <= 0 || !size_ring(c, kOpFwd, kBatchedThreads / tg, room, &smem, true)) return p;
  p.kind = kPlanRegTile;
  p.c = c;
  p.cpt = cpt;
  p.grid = (int)(BT < di.sms ? BT : di.sms);
  p.smem = (int64_t)(batched_q_off(c) + (size_t)batched_slots((int)S) * c.row_bytes);
  return p;
}

struct StreamBatchedPlan {
  bool ok = false;
  StreamBatchedCfg c{};
  int grid = 0;
  int64_t smem = 0;
};

// Row-stream batched forward (the shapes the register tile cannot hold): S
// queries in SB = 4, 8 or 16 slots, CPL = 1 or 2 chunks per lane (2 when the
// queries' registers, SB * CPL 16-byte chunks, stay within 16), rows of exactly
// 32 * CPL * K chunks with K = 2 .. 16 warps per token, N <= 32. Whole tokens
// per token stream, as evenly as possible.
StreamBatchedPlan plan_stream_batched(int64_t N, int64_t BT, int64_t D, int64_t S, int dtype,
                                      const DevInfo& di) {
  StreamBatchedPlan p;
  const int es = esize_of(dtype);
  if (!es || N < 1 || N > kStreamBatchedMaxN || S < 1 || S > kStreamBatchedMaxS || D < 1 ||
      D > kMaxD || BT < 1 || BT > INT_MAX)
    return p;
  if ((D * es) % 16) return p;
  const int64_t rc = D * es / 16;
  const int sb = S <= 4 ? 4 : (S <= 8 ? 8 : 16);
  int cpl = 0;
  for (int cand = 2; cand >= 1 && !cpl; cand /= 2) {  // (4 chunks per lane spill)
    if (sb * cand > 16 || rc % (32 * cand)) continue;
    const int64_t k = rc / (32 * cand);
    if (k >= 2 && k <= 16) cpl = cand;
  }
  if (!cpl) return p;
  const int64_t kw = rc / (32 * cpl);
  const int64_t max_streams = kStreamBatchedThreads / 32 / kw;
  const int64_t g0 = BT < di.sms ? BT : di.sms;
  const int64_t t = (BT + g0 - 1) / g0;
  const int64_t k = (t + max_streams - 1) / max_streams;
  int64_t streams = (t + k - 1) / k;
  if (streams > 8) streams = 8;  // named barrier ids 1..8
  const int64_t qg = stream_batched_qg(cpl);
  const int64_t ngrp = (S + qg - 1) / qg;
  if (((t + streams - 1) / streams) * N * (1 + ngrp) >= (int64_t)INT_MAX) return p;
  StreamBatchedCfg c{};
  c.BT = BT;
  c.N = (int)N;
  c.D = (int)D;
  c.S = (int)S;
  c.row_chunks = (int)rc;
  c.row_bytes = (int)(D * es);
  c.kw = (int)kw;
  c.cpl = cpl;
  c.sb = sb;
  c.warps = (int)(streams * kw);
  c.ring = 0;
  const int64_t fixed = (int64_t)stream_batched_smem_layout(c).total;
  const int64_t per_row = streams * ((int64_t)c.row_bytes + 8 + 4);
  int64_t ring = (di.max_smem - fixed - 16) / per_row;
  if (ring > 16) ring = 16;
  if (ring < 2) return p;
  c.ring = (int)ring;
  p.smem = (int64_t)stream_batched_smem_layout(c).total;
  if (p.smem > di.max_smem) return p;
  p.c = c;
  p.grid = (int)g0;
  p.ok = true;
  return p;
}

cudaError_t launch_plan_batched(const TilePlan& p, int S, int dtype, const void* v,
                                const void* q, void* out, cudaStream_t st) {
  switch (dtype) {
    case SY_BF16:
      return launch_batched_bf16(p.c, p.grid, p.cpt, S, v, q, out, st);
    case SY_F16:
      return launch_batched_f16(p.c, p.grid, p.cpt, S, v, q, out, st);
    case SY_F32:
      return launch_batched_f32(p.c, p.grid, p.cpt, S, v, q, out, st);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_plan_fwd(const TilePlan& p, int dtype, const void* v, const void* w,
                            int w_dtype, void* out, float* stats, cudaStream_t st) {
  if (p.kind == kPlanRegTile) {
    switch (dtype) {
      case SY_BF16:
        return launch_reg_fwd_bf16(p.c, p.grid, p.cpt, v, w, w_dtype, out, stats, st);
      case SY_F16:
        return launch_reg_fwd_f16(p.c, p.grid, p.cpt, v, w, w_dtype, out, stats, st);
      case SY_F32:
        return launch_reg_fwd_f32(p.c, p.grid, p.cpt, v, w, w_dtype, out, stats, st);
    }
    return cudaErrorInvalidValue;
  }
  return launch_tile_fwd(p.c, p.grid, p.cpt, dtype, v, w, w_dtype, out, stats, st);
}

cudaError_t launch_plan_bwd(const TilePlan& p, int dtype, const void* v, const void* w,
                            int w_dtype, const void* g, const float* stats, void* dv, float* dwp,
                            cudaStream_t st) {
  if (p.kind == kPlanRegTile) {
    switch (dtype) {
      case SY_BF16:
        return launch_reg_bwd_bf16(p.c, p.grid, p.cpt, v, w, w_dtype, g, stats, dv, dwp, st);
      case SY_F16:
        return launch_reg_bwd_f16(p.c, p.grid, p.cpt, v, w, w_dtype, g, stats, dv, dwp, st);
      case SY_F32:
        return launch_reg_bwd_f32(p.c, p.grid, p.cpt, v, w, w_dtype, g, stats, dv, dwp, st);
    }
    return cudaErrorInvalidValue;
  }
  return launch_tile_bwd(p.c, p.grid, p.cpt, dtype, v, w, w_dtype, g, stats, dv, dwp, st);
}

int generic_grid(int64_t BT, const DevInfo& di) {
  const int64_t g = (int64_t)di.sms * 4;
  return (int)(BT < g ? BT : g);
}

int64_t generic_partials(int64_t BT, const DevInfo& di) {
  const int64_t g = (int64_t)di.sms * 2;
  const int64_t p = BT < g ? BT : g;
  return p < 1 ? 1 : p;
}

thread_local char t_last_error[256] = "";

int cuda_status(cudaError_t e, const char* where) {
  if (e == cudaSuccess) return SY_OK;
  snprintf(t_last_error, sizeof(t_last_error), "%s: %s", where, cudaGetErrorString(e));
  return SY_ERR_CUDA;
}

bool generic_fwd_fits(int64_t N, const DevInfo& di) {
  return N <= kGenericMaxN && (N * 8 * 2 + 3 * N) * 4 <= di.max_smem;
}

bool generic_batched_fits(int64_t N, int64_t S, const DevInfo& di) {
  return (N * (S + 1) * 8 + S * N) * 4 <= di.max_smem;
}

}  // namespace
}  // namespace sy

using namespace sy;

extern "C" {

const char* sy_status_string(int status) {
  switch (status) {
    case SY_OK:
      return "ok";
    case SY_ERR_ARG:
      return "invalid argument (shape, size or null pointer)";
    case SY_ERR_DTYPE:
      return "unknown dtype code";
    case SY_ERR_UNSUPPORTED:
      return "shape outside the kernels' limits";
    case SY_ERR_CUDA:
      return t_last_error[0] ? t_last_error : "CUDA error";
    case SY_ERR_DEVICE:
      return "a kernel recorded a device-side error (bounded wait expired)";
    case SY_ERR_SCRATCH:
      return "shape needs more dw scratch than sy_bwd_noalloc's fixed array holds "
             "(partial rows x D > sy_bwd_noalloc_max_floats()); use sy_bwd with a caller buffer";
    default:
      return "unknown status";
  }
}

const char* sy_version(void) { return "switchyard-b200 0.1.0 (sm_100a)"; }

int64_t sy_stats_stride(int64_t N) { return N < 1 ? 0 : stats_stride(N); }

int sy_fwd(const void* v, const void* w, void* out, float* stats, int64_t N, int64_t BT,
           int64_t D, int dtype, int w_dtype, float eps, sy_stream_t stream) {
  if (!esize_of(dtype) || !esize_of(w_dtype)) return SY_ERR_DTYPE;
  if (N < 1 || BT < 0 || D < 0) return SY_ERR_ARG;
  if (BT == 0 || D == 0) return SY_OK;
  if (!v || !w || !out) return SY_ERR_ARG;
  if (D > kMaxD || BT > INT_MAX) return SY_ERR_UNSUPPORTED;
  DevInfo di;
  cudaError_t e = dev_info(&di);
  if (e != cudaSuccess) return cuda_status(e, "sy_fwd: device query");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool aligned = al16(v) && al16(out);
  // The planners size kernels from the shape alone; eps is set here. Order:
  // the re-read row stream (4 KiB rows, any N), the register tile (N <= 9),
  // the row stream (rows up to 4 KiB), the shared-memory tile, generic.
  StreamPlan sp = plan_stream(N, BT, D, dtype, di);
  sp.c.eps = eps;
  if (sp.ok && sp.c.reread && aligned) {
    e = launch_stream_fwd(sp.c, sp.grid, sp.cpl, dtype, v, w, w_dtype, out, stats, false, st);
    return cuda_status(e, "sy_fwd: stream kernel launch");
  }
  TilePlan p = plan_tile(kOpFwd, N, BT, D, dtype, di);
  p.c.eps = eps;
  if (p.kind == kPlanRegTile && aligned) {
    e = launch_plan_fwd(p, dtype, v, w, w_dtype, out, stats, st);
    return cuda_status(e, "sy_fwd: register-tile kernel launch");
  }
  if (sp.ok && aligned) {
    e = launch_stream_fwd(sp.c, sp.grid, sp.cpl, dtype, v, w, w_dtype, out, stats, false, st);
    return cuda_status(e, "sy_fwd: stream kernel launch");
  }
  if (p.kind != kPlanGeneric && aligned) {
    e = launch_plan_fwd(p, dtype, v, w, w_dtype, out, stats, st);
    return cuda_status(e, "sy_fwd: tile kernel launch");
  }
  if (!generic_fwd_fits(N, di)) return SY_ERR_UNSUPPORTED;
  e = launch_generic_fwd(BT, (int)N, (int)D, dtype, v, w, w_dtype, out, stats,
                         (int)stats_stride(N), eps, generic_grid(BT, di), st);
  return cuda_status(e, "sy_fwd: generic kernel launch");
}

int64_t sy_bwd_partials(int64_t N, int64_t BT, int64_t D, int dtype) {
  if (!esize_of(dtype) || N < 1 || BT < 0 || D < 0) return -SY_ERR_ARG;
  if (BT == 0 || D == 0) return 1;
  DevInfo di;
  if (dev_info(&di) != cudaSuccess) return -SY_ERR_CUDA;
  const TilePlan p = plan_tile(kOpBwd, N, BT, D, dtype, di);
  // register tile and row stream: one row per CTA; shared-memory tile: one
  // row per group
  if (p.kind == kPlanRegTile) return (int64_t)p.grid;
  const StreamBwdPlan sb = plan_stream_bwd(N, BT, D, dtype, di);
  if (sb.ok) return (int64_t)sb.grid;
  if (p.kind != kPlanGeneric) return (int64_t)p.grid * p.c.groups;
  return generic_partials(BT, di);
}

int sy_bwd(const void* v, const void* w, const void* g, const float* stats, void* dv,
           float* dw_partial, int64_t P, int64_t N, int64_t BT, int64_t D, int dtype,
           int w_dtype, float eps, sy_stream_t stream) {
  if (!esize_of(dtype) || !esize_of(w_dtype)) return SY_ERR_DTYPE;
  if (N < 1 || BT < 0 || D < 0 || P < 1) return SY_ERR_ARG;
  if (P != sy_bwd_partials(N, BT, D, dtype)) return SY_ERR_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (D == 0) return SY_OK;
  if (!dw_partial) return SY_ERR_ARG;
  if (BT == 0) {
    return cuda_status(cudaMemsetAsync(dw_partial, 0, (size_t)P * D * sizeof(float), st),
                       "sy_bwd: zero dw_partial");
  }
  if (!v || !w || !g || !stats || !dv) return SY_ERR_ARG;
  if (D > kMaxD || BT > INT_MAX) return SY_ERR_UNSUPPORTED;
  DevInfo di;
  cudaError_t e = dev_info(&di);
  if (e != cudaSuccess) return cuda_status(e, "sy_bwd: device query");
  // Order: the register tile (N <= 16, rows up to 4 KiB), the row stream
  // (rows of 128 * K chunks, N <= 64), the shared-memory tile, generic.
  TilePlan p = plan_tile(kOpBwd, N, BT, D, dtype, di);
  p.c.eps = eps;
  const bool aligned = al16(v) && al16(g) && al16(stats) && al16(dv) && al16(dw_partial);
  if (p.kind == kPlanRegTile && aligned) {
    e = launch_plan_bwd(p, dtype, v, w, w_dtype, g, stats, dv, dw_partial, st);
    return cuda_status(e, "sy_bwd: register-tile kernel launch");
  }
  const StreamBwdPlan sb = plan_stream_bwd(N, BT, D, dtype, di);
  if (sb.ok && aligned) {
    e = launch_stream_bwd(sb.c, sb.grid, dtype, v, w, w_dtype, g, stats, dv, dw_partial, st);
    return cuda_status(e, "sy_bwd: stream kernel launch");
  }
  if (p.kind != kPlanGeneric && aligned) {
    e = launch_plan_bwd(p, dtype, v, w, w_dtype, g, stats, dv, dw_partial, st);
    return cuda_status(e, "sy_bwd: tile kernel launch");
  }
  if (N > kGenericMaxN || (N * 8 + 3 * N) * 4 > di.max_smem) return SY_ERR_UNSUPPORTED;
  e = launch_generic_bwd(BT, (int)N, (int)D, dtype, v, w, w_dtype, g, stats, (int)stats_stride(N),
                         dv, dw_partial, (int)P, eps, st);
  return cuda_status(e, "sy_bwd: generic kernel launch");
}

int sy_dw_reduce(const float* dw_partial, int64_t P, int64_t D, void* dw, int dw_dtype,
                 sy_stream_t stream) {
  if (!esize_of(dw_dtype)) return SY_ERR_DTYPE;
  if (P < 1 || D < 0) return SY_ERR_ARG;
  if (D == 0) return SY_OK;
  if (!dw_partial || !dw) return SY_ERR_ARG;
  if (D > kMaxD) return SY_ERR_UNSUPPORTED;
  const cudaError_t e =
      launch_dw_reduce(dw_partial, P, D, dw, dw_dtype, SY_TUNE_PDL != 0,
                       static_cast<cudaStream_t>(stream));
  return cuda_status(e, "sy_dw_reduce: launch");
}

int sy_dw_reduce_gain(const float* dw_partial, int64_t P, int64_t D, const void* w, const void* g,
                      void* dw, void* dg, int wg_dtype, sy_stream_t stream) {
  if (!esize_of(wg_dtype)) return SY_ERR_DTYPE;
  if (P < 1 || D < 0) return SY_ERR_ARG;
  if (D == 0 || (!dw && !dg)) return SY_OK;
  if (!dw_partial || !w || !g) return SY_ERR_ARG;
  if (D > kMaxD) return SY_ERR_UNSUPPORTED;
  const cudaError_t e =
      launch_dw_reduce(dw_partial, P, D, dw, wg_dtype, SY_TUNE_PDL != 0,
                       static_cast<cudaStream_t>(stream), w, g, dg);
  return cuda_status(e, "sy_dw_reduce_gain: launch");
}

int sy_fwd_batched(const void* v, const void* queries, void* out, int64_t N, int64_t BT, int64_t D,
                   int64_t S, int dtype, float eps, sy_stream_t stream) {
  if (!esize_of(dtype)) return SY_ERR_DTYPE;
  if (N < 1 || BT < 0 || D < 0 || S < 1) return SY_ERR_ARG;
  if (BT == 0 || D == 0) return SY_OK;
  if (!v || !queries || !out) return SY_ERR_ARG;
  if (D > kMaxD || BT > INT_MAX || S > INT_MAX) return SY_ERR_UNSUPPORTED;
  if (S == 1) return sy_fwd(v, queries, out, nullptr, N, BT, D, dtype, dtype, eps, stream);
  DevInfo di;
  cudaError_t e = dev_info(&di);
  if (e != cudaSuccess) return cuda_status(e, "sy_fwd_batched: device query");
  TilePlan bp = plan_batched(N, BT, D, S, dtype, di);
  bp.c.eps = eps;
  if (bp.kind == kPlanRegTile && al16(v) && al16(queries) && al16(out)) {
    e = launch_plan_batched(bp, (int)S, dtype, v, queries, out, static_cast<cudaStream_t>(stream));
    return cuda_status(e, "sy_fwd_batched: register-tile kernel launch");
  }
  StreamBatchedPlan sb = plan_stream_batched(N, BT, D, S, dtype, di);
  sb.c.eps = eps;
  if (sb.ok && al16(v) && al16(queries) && al16(out)) {
    e = launch_stream_batched(sb.c, sb.grid, dtype, v, queries, out,
                              static_cast<cudaStream_t>(stream));
    return cuda_status(e, "sy_fwd_batched: stream kernel launch");
  }
  if (!generic_batched_fits(N, S, di)) return SY_ERR_UNSUPPORTED;
  e = launch_generic_batched(BT, (int)N, (int)D, (int)S, dtype, nullptr, 0, v, queries, out, eps,
                             generic_grid(BT, di), static_cast<cudaStream_t>(stream));
  return cuda_status(e, "sy_fwd_batched: generic kernel launch");
}

int sy_fwd_batched_stats(const void* v, const void* queries, void* out, float* mstats, int raw,
                         int64_t N, int64_t BT, int64_t D, int64_t S, int dtype, float eps,
                         sy_stream_t stream) {
  if (!esize_of(dtype)) return SY_ERR_DTYPE;
  if (N < 1 || BT < 0 || D < 0 || S < 1 || (raw != 0 && raw != 1)) return SY_ERR_ARG;
  if (BT == 0 || D == 0) return SY_OK;
  if (!v || !queries || !out || !mstats) return SY_ERR_ARG;
  if (D > kMaxD || BT > INT_MAX || S > INT_MAX) return SY_ERR_UNSUPPORTED;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  DevInfo di;
  cudaError_t e = dev_info(&di);
  if (e != cudaSuccess) return cuda_status(e, "sy_fwd_batched_stats: device query");
  const bool aligned = al16(v) && al16(queries) && al16(out) && al8(mstats);
  TilePlan bp = plan_batched(N, BT, D, S, dtype, di);
  bp.c.eps = eps;
  bp.c.mstats = mstats;
  bp.c.raw = raw;
  if (bp.kind == kPlanRegTile && aligned) {
    e = launch_plan_batched(bp, (int)S, dtype, v, queries, out, st);
    return cuda_status(e, "sy_fwd_batched_stats: register-tile kernel launch");
  }
  StreamBatchedPlan sb = plan_stream_batched(N, BT, D, S, dtype, di);
  sb.c.eps = eps;
  sb.c.mstats = mstats;
  sb.c.raw = raw;
  if (sb.ok && aligned) {
    e = launch_stream_batched(sb.c, sb.grid, dtype, v, queries, out, st);
    return cuda_status(e, "sy_fwd_batched_stats: stream kernel launch");
  }
  if (!generic_batched_fits(N, S, di) || !al8(mstats)) return SY_ERR_UNSUPPORTED;
  e = launch_generic_batched(BT, (int)N, (int)D, (int)S, dtype, mstats, raw, v, queries, out, eps,
                             generic_grid(BT, di), st);
  return cuda_status(e, "sy_fwd_batched_stats: generic kernel launch");
}

int64_t sy_bwd_batched_partials(int64_t N, int64_t BT, int64_t D, int64_t S, int dtype) {
  if (!esize_of(dtype) || N < 1 || BT < 0 || D < 0 || S < 1) return -SY_ERR_ARG;
  if (BT == 0 || D == 0) return 1;
  DevInfo di;
  if (dev_info(&di) != cudaSuccess) return -SY_ERR_CUDA;
  // register tile: one CTA per SM for the staged kernel, one or two for the
  // half-pass kernel as its shared memory (its dq columns) allows; generic: two
  const int rc = reg_bwd_batched_ctas_per_sm((int)N, (int)D, (int)S, dtype, di.max_smem);
  const int64_t g = (int64_t)di.sms * (rc > 0 ? rc : 2);
  return BT < g ? BT : g;
}

int sy_bwd_batched(const void* v, const void* queries, const void* g, void* dv,
                   float* dq_partial, int64_t P, int64_t N, int64_t BT, int64_t D,
                   int64_t S, int dtype, float eps, sy_stream_t stream) {
  if (!esize_of(dtype)) return SY_ERR_DTYPE;
  if (N < 1 || BT < 0 || D < 0 || S < 1 || P < 1) return SY_ERR_ARG;
  if (P != sy_bwd_batched_partials(N, BT, D, S, dtype)) return SY_ERR_ARG;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (D == 0) return SY_OK;
  if (!dq_partial) return SY_ERR_ARG;
  if (BT == 0)
    return cuda_status(cudaMemsetAsync(dq_partial, 0, (size_t)P * S * D * sizeof(float), st),
                       "sy_bwd_batched: zero dq_partial");
  if (!v || !queries || !g || !dv) return SY_ERR_ARG;
  if (S > 16) return SY_ERR_UNSUPPORTED;
  if (D > kMaxD || BT > INT_MAX) return SY_ERR_UNSUPPORTED;
  DevInfo di;
  cudaError_t e = dev_info(&di);
  if (e != cudaSuccess) return cuda_status(e, "sy_bwd_batched: device query");
  const int variant = reg_bwd_batched_variant((int)N, (int)D, (int)S, dtype, di.max_smem);
  if (variant > 0 && al16(v) && al16(queries) && al16(g) && al16(dv) && al16(dq_partial)) {
    e = launch_reg_bwd_batched(BT, (int)N, (int)D, (int)S, dtype, v, queries, g, dv, dq_partial,
                               (int)P, eps, variant, st);
    return cuda_status(e, "sy_bwd_batched: register-tile kernel launch");
  }
  if (bwd_batched_smem((int)N, (int)S) > (size_t)di.max_smem) return SY_ERR_UNSUPPORTED;
  e = launch_bwd_batched(BT, (int)N, (int)D, (int)S, dtype, v, queries, g, dv, dq_partial, (int)P,
                         eps, st);
  return cuda_status(e, "sy_bwd_batched: kernel launch");
}

int sy_stage_partial(const void* partial, const void* out, void* new_partial, void* arena_slot,
                     int64_t numel, int dtype, sy_stream_t stream) {
  if (!esize_of(dtype)) return SY_ERR_DTYPE;
  if (numel < 0) return SY_ERR_ARG;
  if (numel == 0) return SY_OK;
  if (!partial || !out || !arena_slot) return SY_ERR_ARG;
  DevInfo di;
  cudaError_t e = dev_info(&di);
  if (e != cudaSuccess) return cuda_status(e, "sy_stage_partial: device query");
  const int es = esize_of(dtype);
  const bool vec16 = (numel * es) % 16 == 0 && al16(partial) && al16(out) && al16(arena_slot) &&
                     (new_partial == nullptr || al16(new_partial));
  const int64_t work = vec16 ? numel * es / 16 : numel;
  const int64_t cap = (int64_t)di.sms * 8;  // 8 CTAs of 256 threads per SM
  const int64_t blocks = (work + 255) / 256;
  e = launch_stage(numel, dtype, partial, out, new_partial, arena_slot, vec16,
                   (int)(blocks < cap ? blocks : cap), static_cast<cudaStream_t>(stream));
  return cuda_status(e, "sy_stage_partial: kernel launch");
}

int sy_merge_stats(const void* o1, const float* ms1, const void* o2, const float* ms2, void* o,
                   float* ms, int normalize, int64_t R, int64_t D, int dtype,
                   sy_stream_t stream) {
  if (!esize_of(dtype)) return SY_ERR_DTYPE;
  if (R < 0 || D < 0 || (normalize != 0 && normalize != 1)) return SY_ERR_ARG;
  if (R == 0) return SY_OK;
  if (!o1 || !ms1 || !o2 || !ms2 || (D > 0 && !o)) return SY_ERR_ARG;
  if (!al8(ms1) || !al8(ms2) || (ms && !al8(ms))) return SY_ERR_ARG;
  if (D > kMaxD) return SY_ERR_UNSUPPORTED;
  DevInfo di;
  cudaError_t e = dev_info(&di);
  if (e != cudaSuccess) return cuda_status(e, "sy_merge_stats: device query");
  const int vec16 = (D * esize_of(dtype)) % 16 == 0 && al16(o1) && al16(o2) && al16(o);
  const int64_t cap = (int64_t)di.sms * 8;  // one row per CTA, 8 CTAs per SM in flight
  e = launch_merge(R, (int)D, dtype, o1, ms1, o2, ms2, o, ms, normalize, vec16,
                   (int)(R < cap ? R : cap), static_cast<cudaStream_t>(stream));
  return cuda_status(e, "sy_merge_stats: kernel launch");
}

int sy_speed_of_light(const void* v, void* out, int64_t N, int64_t BT, int64_t D, int dtype,
                      sy_stream_t stream) {
  if (!esize_of(dtype)) return SY_ERR_DTYPE;
  if (N < 1 || BT < 0 || D < 0) return SY_ERR_ARG;
  if (BT == 0 || D == 0) return SY_OK;
  if (!v || !out) return SY_ERR_ARG;
  if (D > kMaxD || BT > INT_MAX) return SY_ERR_UNSUPPORTED;
  DevInfo di;
  cudaError_t e = dev_info(&di);
  if (e != cudaSuccess) return cuda_status(e, "sy_speed_of_light: device query");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const StreamPlan sp = plan_stream(N, BT, D, dtype, di, /*sol=*/true);
  if (sp.ok && al16(v) && al16(out)) {
    e = launch_stream_fwd(sp.c, sp.grid, sp.cpl, dtype, v, nullptr, SY_F32, out, nullptr, true, st);
    return cuda_status(e, "sy_speed_of_light: stream kernel launch");
  }
  const TilePlan p = plan_tile(kOpSol, N, BT, D, dtype, di);
  if (p.kind != kPlanGeneric && al16(v) && al16(out)) {
    e = launch_tile_sol(p.c, p.grid, p.cpt, dtype, v, out, st);
    return cuda_status(e, "sy_speed_of_light: tile kernel launch");
  }
  e = launch_generic_sol(BT, (int)N, (int)D, dtype, v, out, generic_grid(BT, di), st);
  return cuda_status(e, "sy_speed_of_light: generic kernel launch");
}

int sy_plan_info(int op, int64_t N, int64_t BT, int64_t D, int64_t S, int dtype, int sms,
                 int max_smem, int64_t* out) {
  if (!out) return SY_ERR_ARG;
  if (!esize_of(dtype)) return SY_ERR_DTYPE;
  if (N < 1 || BT < 0 || D < 0 || op < 0 || op > 3) return SY_ERR_ARG;
  DevInfo di;
  if (sms > 0 && max_smem > 0) {
    di.sms = sms;
    di.max_smem = max_smem;
    di.l2 = kAssumedL2Bytes;
  } else {
    const cudaError_t e = dev_info(&di);
    if (e != cudaSuccess) return cuda_status(e, "sy_plan_info: device query");
  }
  const int64_t bt = BT < 1 ? 1 : BT;
  int top = op == 1 ? kOpBwd : (op == 3 ? kOpSol : kOpFwd);
  if (op == 2 && S < 1) return SY_ERR_ARG;
  if (top != kOpBwd && (op != 2 || S == 1)) {
    const StreamPlan sp = plan_stream(N, bt, D, dtype, di, top == kOpSol);
    const bool reg_first = top == kOpFwd && !sp.c.reread &&
                           plan_tile(kOpFwd, N, bt, D, dtype, di).kind == kPlanRegTile;
    if (sp.ok && !reg_first) {
      const int kw = sp.c.kw > 1 ? sp.c.kw : 1;
      out[0] = kPlanStream;
      out[1] = sp.grid;
      out[2] = sp.c.ring;
      out[3] = sp.c.warps / kw;  // token streams per CTA
      out[4] = 32 * kw;          // threads per token stream
      out[5] = sp.cpl;
      out[6] = sp.c.row_bytes;
      out[7] = sp.smem;
      return SY_OK;
    }
  }
  if (top == kOpBwd && plan_tile(kOpBwd, N, bt, D, dtype, di).kind != kPlanRegTile) {
    const StreamBwdPlan sb = plan_stream_bwd(N, bt, D, dtype, di);
    if (sb.ok) {
      out[0] = kPlanStream;
      out[1] = sb.grid;
      out[2] = sb.c.ring;
      out[3] = sb.c.warps / sb.c.kw;  // token streams per CTA
      out[4] = 32 * sb.c.kw;          // threads per token stream
      out[5] = sb.c.cpl;
      out[6] = sb.c.row_bytes;
      out[7] = sb.smem;
      return SY_OK;
    }
  }
  TilePlan p;
  if (op != 2 || S == 1)
    p = plan_tile(top, N, bt, D, dtype, di);
  else
    p = plan_batched(N, bt, D, S, dtype, di);
  if (op == 2 && S > 1 && p.kind != kPlanRegTile) {
    const StreamBatchedPlan sb = plan_stream_batched(N, bt, D, S, dtype, di);
    if (sb.ok) {
      out[0] = kPlanStream;
      out[1] = sb.grid;
      out[2] = sb.c.ring;
      out[3] = sb.c.warps / sb.c.kw;  // token streams per CTA
      out[4] = 32 * sb.c.kw;          // threads per token stream
      out[5] = sb.c.cpl;              // chunks per lane
      out[6] = sb.c.row_bytes;
      out[7] = sb.smem;
      return SY_OK;
    }
  }
  out[0] = p.kind;
  out[1] = p.grid;
  out[2] = p.c.stages;
  out[3] = p.c.groups;
  out[4] = p.c.tg;
  out[5] = p.cpt;
  out[6] = p.c.stage_bytes;
  out[7] = p.smem;
  return SY_OK;
}

int sy_plan_kind(int op, int64_t N, int64_t BT, int64_t D, int64_t S, int dtype) {
  int64_t info[8];
  const int st = sy_plan_info(op, N, BT, D, S, dtype, 0, 0, info);
  return st == SY_OK ? (int)info[0] : -st;
}

int sy_device_error(int* code) {
  if (!code) return SY_ERR_ARG;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e, "sy_device_error: synchronize");
  unsigned int v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v));
  if (e != cudaSuccess) return cuda_status(e, "sy_device_error: read");
  const unsigned int zero = 0;
  e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
  if (e != cudaSuccess) return cuda_status(e, "sy_device_error: clear");
  *code = (int)v;
  return SY_OK;
}

}  // extern "C"
