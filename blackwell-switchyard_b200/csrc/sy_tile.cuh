// sy_tile.cuh -- the TMA-pipelined "token tile" kernel family.
//
// One persistent CTA per SM. Warp 0 is the producer: one elected lane streams
// each token's N source rows (plus, in the backward, the upstream-gradient row
// and the token's saved statistics) from HBM into a ring of shared-memory
// stages with cp.async.bulk, signalling an mbarrier per stage. The remaining
// warps form G consumer groups of TG threads; group g takes every G-th token
// of the CTA, so groups overlap one another's reductions with loads and math.
// Inside a group, thread t owns 16-byte chunks t, t+TG, ... of every row
// (CPT chunks), so a token's row reductions are a per-thread FMA chain, one
// warp reduce-scatter and one named barrier -- v is read from HBM exactly
// once and every row is touched twice from shared memory.
//
// Tokens are assigned statically: CTA b handles tokens b, b+grid, b+2*grid...
// and group g of it the k-th of those with k % G == g. Every reduction has a
// fixed order, so results are bitwise reproducible for a given grid.
#pragma once

#include "sy_common.cuh"

namespace sy {

// Largest source count the tile kernels handle (lane j of a warp owns rows j
// and j+32 during the softmax).
constexpr int kTileMaxN = 64;
// Threads per consumer block in the tile kernels, producer warp excluded.
constexpr int kConsumerThreads = 256;

struct TileCfg {
  long long BT;      // tokens
  int N;             // sources
  int D;             // full row length in elements
  int row_chunks;    // 16-byte chunks per row
  int row_bytes;     // bytes per row (= D * esize)
  int stage_bytes;   // bytes per pipeline stage (multiple of 128)
  int stages;        // S
  int groups;        // G
  int tg;            // threads per consumer group (multiple of 32)
  int stats_stride;  // floats per token in the statistics buffer
  int red_stride;    // floats per consumer warp in one reduction buffer
  int coef_stride;   // floats per consumer warp in the per-source coefficients
  int w_smem;        // register-tile forward: w kept in shared memory (fp32)
  int hold;          // register-tile forward: tile held in the stage (no register copy)
  float eps;
  // batched forward only: per (query, token) (max logit, sum of exp(logit - max))
  // as float pairs [S][BT][2] when non-null, and raw = 1 writes the
  // unnormalised sum_n exp(logit_n - max) v_n instead of the softmax average
  float* mstats;
  int raw;
};

// Per-warp scratch sizes for N sources: the reduction holds 16 values per
// block of 8 rows (forward: dot and sum of squares; backward uses half), the
// coefficients one float4 per source.
__host__ __device__ inline int tile_red_stride(int N) { return 16 * ((N + 7) / 8); }
__host__ __device__ inline int tile_coef_stride(int N) { return 4 * ((N + 7) / 8) * 8; }

// Shared-memory carve-up, identical on host (sizing) and device (pointers).
struct TileSmem {
  size_t stages_off, red_off, coef_off, bar_off, zero_off, w_off, total;
};

__host__ __device__ inline TileSmem tile_smem_layout(const TileCfg& c) {
  TileSmem s;
  const int nwc = c.groups * c.tg / 32;  // consumer warps
  s.stages_off = 0;
  s.red_off = (size_t)c.stages * c.stage_bytes;
  s.coef_off = s.red_off + (size_t)2 * nwc * c.red_stride * sizeof(float);
  s.bar_off = s.coef_off + (size_t)nwc * c.coef_stride * sizeof(float);
  s.zero_off = s.bar_off + (size_t)2 * c.stages * sizeof(uint64_t);  // 16 zero bytes
  s.w_off = s.zero_off + 16;  // fp32 copy of w (w_smem != 0): D floats, 16-byte planes
  s.total = s.w_off + (c.w_smem ? ((size_t)c.D * 4 + 15) / 16 * 16 : 0);
  return s;
}

// Host launchers (defined in sy_tile_fwd.cu / sy_tile_bwd.cu). `cpt` is the
// number of 16-byte chunks per consumer thread per row (1, 2 or 4).
cudaError_t launch_tile_fwd(const TileCfg& c, int grid, int cpt, int dtype, const void* v,
                            const void* w, int w_dtype, void* out, float* stats,
                            cudaStream_t st);
cudaError_t launch_tile_sol(const TileCfg& c, int grid, int cpt, int dtype, const void* v,
                            void* out, cudaStream_t st);
cudaError_t launch_tile_bwd(const TileCfg& c, int grid, int cpt, int dtype, const void* v,
                            const void* w, int w_dtype, const void* g, const float* stats,
                            void* dv, float* dw_partial, cudaStream_t st);

// Register-tile kernels (sy_reg_{bf16,f16,f32}.cu), exact N in 1..16.
#define SY_REG_DECL(dt)                                                                         \
  cudaError_t launch_reg_fwd_##dt(const TileCfg& c, int grid, int cpt, const void* v,          \
                                  const void* w, int w_dtype, void* out, float* stats,          \
                                  cudaStream_t st);                                             \
  cudaError_t launch_reg_bwd_##dt(const TileCfg& c, int grid, int cpt, const void* v,          \
                                  const void* w, int w_dtype, const void* g, const float* stats, \
                                  void* dv, float* dwp, cudaStream_t st);
SY_REG_DECL(bf16)
SY_REG_DECL(f16)
SY_REG_DECL(f32)
#undef SY_REG_DECL

// Generic kernels (sy_generic.cu): any D, any 2-byte/4-byte alignment, N up to
// kGenericMaxN. One CTA per token, two passes over the row (second from L2).
constexpr int kGenericMaxN = 2048;
constexpr int kGenericThreads = 256;
cudaError_t launch_generic_fwd(long long BT, int N, int D, int dtype, const void* v,
                               const void* w, int w_dtype, void* out, float* stats, int stats_stride,
                               float eps, int grid, cudaStream_t st);
cudaError_t launch_generic_sol(long long BT, int N, int D, int dtype, const void* v, void* out,
                               int grid, cudaStream_t st);
cudaError_t launch_generic_bwd(long long BT, int N, int D, int dtype, const void* v,
                               const void* w, int w_dtype, const void* g, const float* stats,
                               int stats_stride, void* dv, float* dw_partial, int P, float eps,
                               cudaStream_t st);
cudaError_t launch_bwd_batched(long long BT, int N, int D, int S, int dtype, const void* v,
                               const void* q, const void* g, void* dv, float* dq_partial, int P,
                               float eps, cudaStream_t st);
size_t bwd_batched_smem(int N, int S);
bool reg_bwd_batched_fits(int N, int D, int S, int dtype, int max_smem);
int reg_bwd_batched_ctas_per_sm(int N, int D, int S, int dtype, int max_smem);
int reg_bwd_batched_variant(int N, int D, int S, int dtype, int max_smem);
cudaError_t launch_stage(long long numel, int dtype, const void* partial, const void* out,
                         void* new_partial, void* arena, bool vec16, int grid, cudaStream_t st);
cudaError_t launch_reg_bwd_batched(long long BT, int N, int D, int S, int dtype, const void* v,
                                   const void* q, const void* g, void* dv, float* dq_partial,
                                   int P, float eps, int variant, cudaStream_t st);
cudaError_t launch_merge(long long R, int D, int dtype, const void* o1, const float* ms1,
                         const void* o2, const float* ms2, void* o, float* ms, int normalize,
                         int vec16, int grid, cudaStream_t st);
cudaError_t launch_generic_batched(long long BT, int N, int D, int S, int dtype, float* mstats,
                                   int raw, const void* v,
                                   const void* q, void* out, float eps, int grid, cudaStream_t st);

// Fixed-order column reduction of dw partials (sy_tile_bwd.cu); with gw and gg
// (w and g of q = w * g) the result is split into dw = dq * g and dg = dq * w.
cudaError_t launch_dw_reduce(const float* part, long long P, long long D, void* dw, int dw_dtype,
                             bool pdl, cudaStream_t st, const void* gw = nullptr,
                             const void* gg = nullptr, void* dg = nullptr);

}  // namespace sy
