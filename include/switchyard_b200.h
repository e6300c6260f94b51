/*
 * switchyard_b200.h -- C ABI of the B200 (sm_100a) Block AttnRes operator.
 *
 * The operator, per token (b, t), over N source rows v[n, b, t, :] of length D
 * and one query w[D]:
 *
 *     r_n     = 1 / sqrt(mean_d v[n,d]^2 + eps)        inverse RMS of source n
 *     logit_n = r_n * sum_d w[d] v[n,d]                 no 1/sqrt(D) scale
 *     alpha   = softmax_n(logit)                        over the source axis
 *     out[d]  = sum_n alpha_n v[n,d]                    raw (unnormalised) v
 *
 * Everything here is plain C: raw device pointers, element counts, a dtype
 * code and a CUDA stream passed as `void*` (a cudaStream_t; NULL means the
 * legacy default stream). No entry point allocates device memory; callers own
 * every buffer. Launches are asynchronous on the given stream. Every function
 * returns SY_OK or a nonzero status (see sy_status_string); none of them
 * traps or aborts on bad input.
 *
 * Layouts (all row-major, contiguous):
 *   v      [N, BT, D]      BT = B*T tokens; element (n,tok,d) at (n*BT+tok)*D+d
 *   out    [BT, D]         dtype of v
 *   w      [D]             any of the three dtypes (w_dtype)
 *   stats  [BT, SW] fp32   SW = sy_stats_stride(N); per token:
 *                          logit[0..N), r[0..N), max logit m, logsumexp lse
 *   g      [BT, D]         upstream gradient, dtype of v
 *   dv     [N, BT, D]      dtype of v
 *   dw_partial [P, D] fp32 P = sy_bwd_partials(...) rows, reduced by
 *                          sy_dw_reduce in a fixed order (deterministic)
 *   queries [S, D], out_batched [S, BT, D]   dtype of v
 *
 * The reference this replaces is Python/Triton (sabdulmajid/blackwell-switchyard,
 * src/switchyard/triton_op.py); it has no C interface of its own. Each entry
 * point below names the reference function whose job it takes over.
 */
#ifndef SWITCHYARD_B200_H
#define SWITCHYARD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes */
#define SY_BF16 0
#define SY_F16 1
#define SY_F32 2

/* status codes */
#define SY_OK 0
#define SY_ERR_ARG 1         /* bad shape, size or null pointer              */
#define SY_ERR_DTYPE 2       /* unknown dtype code                           */
#define SY_ERR_UNSUPPORTED 3 /* shape outside every kernel's limits          */
#define SY_ERR_CUDA 4        /* a CUDA runtime call or launch failed         */
#define SY_ERR_DEVICE 5      /* a kernel reported a device-side error word   */
#define SY_ERR_SCRATCH 6     /* shape needs more than sy_bwd_noalloc's fixed
                                scratch (sy_bwd_noalloc_max_floats floats)  */

typedef void* sy_stream_t; /* a cudaStream_t */

/* Exported symbols; everything else in the library is hidden. */
#if defined(__GNUC__)
#define SY_API __attribute__((visibility("default")))
#else
#define SY_API
#endif

/* Human-readable text for a status code (static storage). */
SY_API const char* sy_status_string(int status);

/* Library version string (static storage). */
SY_API const char* sy_version(void);

/* Floats per token in the statistics buffer written by sy_fwd:
 * round_up(2*N + 2, 4). */
SY_API int64_t sy_stats_stride(int64_t N);

/*
 * Forward. Replaces _BlockAttnResTriton.forward and its kernels
 * _fwd_resident/_fwd_tiled (src/switchyard/triton_op.py:504-536, :50-117).
 * `stats` may be NULL (inference); when given it must hold BT*sy_stats_stride(N)
 * floats and is what sy_bwd reads.
 */
SY_API int sy_fwd(const void* v, const void* w, void* out, float* stats, int64_t N,
           int64_t BT, int64_t D, int dtype, int w_dtype, float eps,
           sy_stream_t stream);

/*
 * Number of dw partial rows sy_bwd writes for this shape on the current
 * device (>= 1). Replaces nothing in the reference: its backward used one
 * fp32 accumulator with atomics (src/switchyard/triton_op.py:547-550, :264).
 */
SY_API int64_t sy_bwd_partials(int64_t N, int64_t BT, int64_t D, int dtype);

/*
 * Backward from saved statistics. Replaces _BlockAttnResTriton.backward with
 * _bwd_resident / _bwd_stats / _bwd_apply (src/switchyard/triton_op.py:538-589,
 * :194-375). Writes every element of dv and every row of dw_partial
 * (P = sy_bwd_partials rows of D fp32); no zero-fill is needed beforehand.
 */
SY_API int sy_bwd(const void* v, const void* w, const void* g, const float* stats,
           void* dv, float* dw_partial, int64_t P, int64_t N, int64_t BT,
           int64_t D, int dtype, int w_dtype, float eps, sy_stream_t stream);

/*
 * dw[d] = sum_{p=0..P-1} dw_partial[p, d], summed in a fixed order and
 * written in dw_dtype. Replaces the reference's torch.zeros fill and the
 * dw.to(w.dtype) cast (src/switchyard/triton_op.py:550, :563, :589).
 */
SY_API int sy_dw_reduce(const float* dw_partial, int64_t P, int64_t D, void* dw,
                 int dw_dtype, sy_stream_t stream);

/*
 * sy_dw_reduce with the module's gain folded in. BlockAttnResTriton's forward
 * queries with q = w * g (src/switchyard/triton_op.py:605-609), so autograd
 * turns the reduced dq into dw = dq * g and dg = dq * w with two more
 * elementwise kernels; this call does the reduction and both products in one
 * launch, with the same roundings (dq rounded to wg_dtype first, each product
 * rounded to wg_dtype). w, g, dw, dg: [D] of wg_dtype; dw or dg may be NULL
 * (that gradient is not written).
 */
SY_API int sy_dw_reduce_gain(const float* dw_partial, int64_t P, int64_t D, const void* w,
                      const void* g, void* dw, void* dg, int wg_dtype, sy_stream_t stream);

/*
 * Batched-query forward, output only: out[s] = forward(v, queries[s]).
 * Replaces block_attn_res_batched and _fwd_batched_resident
 * (src/switchyard/triton_op.py:438-501, :378-414), including the shapes the
 * reference sent to its per-query fallback loop.
 */
SY_API int sy_fwd_batched(const void* v, const void* queries, void* out, int64_t N,
                   int64_t BT, int64_t D, int64_t S, int dtype, float eps,
                   sy_stream_t stream);

/*
 * Batched forward that also returns the merge statistics: as sy_fwd_batched,
 * plus mstats[(s * BT + tok) * 2 + {0, 1}] = (m, l) = (max_n logit_{s,n},
 * sum_n exp(logit_{s,n} - m)) in fp32 (8-byte aligned). raw = 0 writes the
 * softmax average (the block_attn_res_batched output); raw = 1 writes the
 * unnormalised o = sum_n exp(logit_{s,n} - m) v_n, so (out, m, l) is the
 * (o, m, ell) triple of attn_with_stats (src/switchyard/reference.py:195-216)
 * for each query. S >= 1 (S = 1 is attn_with_stats for one query). The
 * reference's batched API returns no statistics (README.md:63-70); this is
 * the first half of its "complete the batched training contract" item
 * (PROJECT_STATE.md:74-75).
 */
SY_API int sy_fwd_batched_stats(const void* v, const void* queries, void* out,
                                float* mstats, int raw, int64_t N, int64_t BT,
                                int64_t D, int64_t S, int dtype, float eps,
                                sy_stream_t stream);

/* Number of fp32 dq partial rows (each S * D floats) sy_bwd_batched expects
 * for a shape on the current device (>= 1), or -status. */
SY_API int64_t sy_bwd_batched_partials(int64_t N, int64_t BT, int64_t D,
                                       int64_t S, int dtype);

/*
 * Backward of the batched forward (sy_fwd_batched, or sy_fwd_batched_stats
 * with raw = 0): the second half of the batched training contract the
 * reference lacks (src/switchyard/triton_op.py:475-479 raises instead).
 * g: gradient of out, [S, BT, D] in v's dtype. Writes dv [N, BT, D] in v's
 * dtype and P = sy_bwd_batched_partials(..) fp32 partial rows dq_partial
 * [P, S, D]; sy_dw_reduce(dq_partial, P, S * D, dq, dtype) then gives dq
 * [S, D] in a fixed summation order. The dot products and the softmax are
 * recomputed from v and the queries in one pass per token, so nothing is
 * saved by the forward. S <= 16.
 */
SY_API int sy_bwd_batched(const void* v, const void* queries, const void* g,
                          void* dv, float* dq_partial, int64_t P, int64_t N,
                          int64_t BT, int64_t D, int64_t S, int dtype, float eps,
                          sy_stream_t stream);

/*
 * Online-softmax merge of two partial results over disjoint source groups,
 * R rows of D (merge_online_softmax, src/switchyard/reference.py:219-233):
 * m = max(m1, m2), s_i = exp(m_i - m), o = o1 s1 + o2 s2, l = l1 s1 + l2 s2,
 * with (m, l) pairs per row in ms1 / ms2 / ms (fp32, 8-byte aligned; ms may
 * be NULL). normalize = 1 writes o / l (the finished output) instead of o.
 * o must not alias o1 or o2.
 */
SY_API int sy_merge_stats(const void* o1, const float* ms1, const void* o2,
                          const float* ms2, void* o, float* ms, int normalize,
                          int64_t R, int64_t D, int dtype, sy_stream_t stream);

/*
 * The decoder's arena staging step in one pass: new_partial = partial + out
 * (fp32 add, one rounding to dtype) written to new_partial and to arena_slot,
 * numel elements each. Replaces `partial = partial + out` followed by
 * `arena[len(blocks)].copy_(partial)` (src/switchyard/model.py:532-535):
 * 4 slab passes in one launch instead of 5 in two. new_partial may be NULL
 * (only the arena slot is written). No buffer may overlap another.
 */
SY_API int sy_stage_partial(const void* partial, const void* out, void* new_partial,
                            void* arena_slot, int64_t numel, int dtype,
                            sy_stream_t stream);

/*
 * Speed-of-light ceiling: out[tok, d] = sum_n v[n, tok, d]. Same bytes and
 * access pattern as sy_fwd without the softmax. Replaces speed_of_light /
 * _speed_of_light (src/switchyard/triton_op.py:153-191).
 */
SY_API int sy_speed_of_light(const void* v, void* out, int64_t N, int64_t BT,
                      int64_t D, int dtype, sy_stream_t stream);

/*
 * Which kernel family sy_fwd / sy_bwd / sy_fwd_batched would launch for a
 * shape on the current device, without launching: 1 = register-tile kernel
 * (exact N, TMA-pipelined), 2 = shared-memory tile kernel (run-time N,
 * TMA-pipelined), 3 = row-stream kernel (one warp per token, online softmax,
 * forward only), 0 = generic (any size/alignment) kernel, <0 = -status.
 * `op` is 0 forward, 1 backward, 2 batched (S queries), 3 speed of light.
 * Used by tests to pin dispatch, like the reference's _launch_config tests
 * (src/switchyard/triton_op.py:130-150, :267-276, :420-435).
 */
SY_API int sy_plan_kind(int op, int64_t N, int64_t BT, int64_t D, int64_t S,
                        int dtype);

/*
 * The full launch plan for a shape on a device with `sms` multiprocessors
 * and `max_smem` bytes of opt-in shared memory per block (pass 0, 0 for the
 * current device). Writes out[8] = {kind (as sy_plan_kind), grid, pipeline
 * stages, consumer groups, threads per group, 16-byte chunks per thread per
 * row, bytes per stage, dynamic shared memory bytes}; for the row-stream
 * kind: {3, grid, row buffers per warp, warps per CTA, 32, chunks per lane,
 * bytes per row, shared memory bytes}. No reference counterpart; exposes the
 * planner to tests.
 */
SY_API int sy_plan_info(int op, int64_t N, int64_t BT, int64_t D, int64_t S,
                        int dtype, int sms, int max_smem, int64_t* out);

/*
 * Backward plus dw reduction for callers that cannot allocate device memory
 * (a plugin in a host framework that owns all device memory, or a
 * latency-critical loop that must not allocate). Same arguments and results as
 * sy_bwd followed by sy_dw_reduce, but the fp32 dw partial rows live in a
 * fixed 8 MiB array inside the library instead of a caller buffer: shapes with
 * sy_bwd_partials(N, BT, D, dtype) * D > sy_bwd_noalloc_max_floats() fail with
 * SY_ERR_SCRATCH. The first call on a device looks the array up (make it before
 * any stream capture); all calls on a device share the array, so calls that
 * overlap on the GPU race. Allocates nothing. No counterpart in the reference.
 */
SY_API int sy_bwd_noalloc(const void* v, const void* w, const void* g,
                          const float* stats, void* dv, void* dw, int64_t N,
                          int64_t BT, int64_t D, int dtype, int w_dtype,
                          float eps, sy_stream_t stream);

/* Capacity of sy_bwd_noalloc's scratch array, in fp32 values. No counterpart
 * in the reference. */
SY_API int64_t sy_bwd_noalloc_max_floats(void);

/*
 * Cross-GPU sum of token-sharded dw, fused with the fixed-order reduction of
 * the rank's partial rows (one call per rank, each on its own GPU). Replaces
 * the data-parallel gradient all-reduce of w that the reference leaves to DDP
 * (bench/bench_ddp.py:49,65) together with the sy_dw_reduce of each rank; the
 * op itself has no multi-GPU code.
 *
 * dw_partial: this rank's [P, L] fp32 partial rows (sy_bwd's dw_partial, L = D;
 * or sy_bwd_batched's, L = S * D), written by earlier work on `stream` (the
 * kernel is a programmatic dependent launch of it).
 * Every rank owns a buffer that all ranks can address (NVLink peer mappings) of
 * sy_dw_exchange_bytes(L, world) bytes at byte offset buf_off (8-byte aligned)
 * from its base, zeroed before the first call; peer_bases is a DEVICE array of
 * `world` 64-bit addresses, entry r = rank r's buffer base. The kernel sums the
 * rank's rows in sy_dw_reduce's order, stores each column as one 8-byte word
 * (fp32 value, tag) into every other rank's buffer, waits in its own buffer for
 * every other rank's words of this tag (bounded by wait_limit_ns; 0 means 2 s),
 * then writes dw[L] in dw_dtype = sum over ranks 0..world-1, in that order --
 * bitwise the same on every rank, and bitwise an all-gather of the ranks'
 * sy_dw_reduce results added in rank order in fp32. Tags start at 1 and
 * increase by one per call, the same sequence on every rank.
 *
 * A wait that runs out does not hang: the block's dw values are NaN, the
 * device error word gets bit 1 (sy_device_error) and, if fail_word is not
 * NULL, the tag is stored there (any device-visible memory; mapped pinned host
 * memory lets the host see it without a synchronisation). timing, if not NULL,
 * is 8 device uint64 counters that block 0 adds to on every call: calls; total
 * and largest nanoseconds from its pushes to the last peer word; total
 * nanoseconds from the kernel's start to the end of its sum; then the totals of
 * its phases: the partial-row sum, the pushes, the wait with the rank-order sum
 * and the output store (the eighth is unused). Plain peer stores and local
 * loads only (no multicast).
 */
SY_API int sy_dw_exchange(const float* dw_partial, int64_t P, int64_t L,
                          const void* peer_bases, int world, int rank, int64_t buf_off,
                          uint32_t tag, void* dw, int dw_dtype, uint64_t wait_limit_ns,
                          unsigned long long* timing, unsigned int* fail_word,
                          sy_stream_t stream);

/* Bytes of each rank's sy_dw_exchange buffer for L columns and `world` ranks:
 * two slots of world * L 8-byte words, or -status. No reference counterpart. */
SY_API int64_t sy_dw_exchange_bytes(int64_t L, int world);

/*
 * Reads the device-side error word of the current device and clears it.
 * Synchronises the device. Bit 1: a kernel's bounded wait ran out; bit 2: a
 * kernel refused an inconsistent launch plan. Writes 0 to *code when no error
 * was recorded.
 */
SY_API int sy_device_error(int* code);

#ifdef __cplusplus
}
#endif

#endif /* SWITCHYARD_B200_H */
