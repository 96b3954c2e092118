/*
 * moe_b200.h — C ABI of the B200-native (sm_100a) fused MoE MLP.
 *
 * The op is the expert MLP of an sglang-style MoE layer:
 *
 *     out = grouped_matmul(x, w13) -> silu(gate) * up -> grouped_matmul(., w2)
 *
 * Reference interface this library replaces (CrDem/mail, Python + Triton):
 *   - fused_moe_mlp(x, w13, w2, group_sizes, BLOCK_M, ...)  fused_moe_mlp_triton.py:121-160
 *   - build_tile_schedule(group_sizes, num_tokens, BLOCK_M)  fused_moe_mlp_triton.py:91-119
 *   - the sglang call site fused_moe_mlp(hidden_states, w13_weight, w2_weight,
 *     expert_tokens)                                           unquant_diff.txt:13-18
 * The top-k entry point (moe_fused_experts) implements the sglang fused_experts-style call
 * fused_moe_mlp(hidden_states, w13, w2, topk_weights, topk_ids, [scales]); the
 * reference has no routing/align/quant/combine code, so those stages follow the
 * semantics documented beside each declaration.
 *
 * Conventions
 *   - All pointers are device pointers unless stated otherwise; sizes are
 *     element counts. No compute entry point allocates device memory: callers
 *     pass a workspace sized by the matching *_workspace_size() query (or,
 *     for moe_align_static, none). The one allocating call is
 *     moe_ipc_malloc, the expert-parallel set-up helper that creates the
 *     CUDA-IPC-shareable buffers peers map.
 *   - Every call is asynchronous on `stream` (a cudaStream_t, NULL = legacy
 *     default stream) and never synchronises the device. Kernels are launched
 *     with programmatic dependent launch (MOE_OPT_PDL) and each waits for the
 *     work queued before it on the stream before touching memory, so ordering
 *     against the caller's own kernels is plain stream order.
 *   - Return value: MOE_OK or a moe_status_t; moe_last_error() returns a
 *     thread-local message for the last failing call of this thread.
 *   - Weight layout ("(E, K, N)" logical, K-major physical): w13 is stored as
 *     [E, 2I, H] row-major (row n of expert e holds the H weights of output
 *     column n; rows [0, I) = gate, [I, 2I) = up) which is the reference's
 *     logical w13[E, H, 2I] viewed through transpose(1, 2) (kernel_bench.py:229-235).
 *     w2 is stored as [E, H, I] row-major (the reference's logical w2[E, I, H]).
 *   - Device-side failures (a pipeline wait that exceeded its time limit) are
 *     latched in a device flag read by moe_get_device_error().
 */
#ifndef MOE_B200_H_
#define MOE_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MOE_API __attribute__((visibility("default")))
#else
#define MOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  MOE_OK = 0,
  MOE_ERR_INVALID_ARG = 1,  /* bad shape / dtype / pointer / alignment */
  MOE_ERR_UNSUPPORTED = 2,  /* valid request the library does not implement */
  MOE_ERR_CUDA = 3,         /* a CUDA runtime or driver call failed */
  MOE_ERR_WORKSPACE = 4,    /* workspace too small */
  MOE_ERR_DEVICE = 5        /* device-side error flag was set (timeout) */
} moe_status_t;

typedef enum {
  MOE_F32 = 0,
  MOE_F16 = 1,
  MOE_BF16 = 2,
  MOE_I8 = 3,
  MOE_I32 = 4,
  MOE_I64 = 5
} moe_dtype_t;

/* GEMM2 epilogue modes (moe_gemm2). */
typedef enum {
  MOE_EPI_STORE_ROWS = 0,   /* out[row] = acc, rows in schedule order (pre-routed form) */
  MOE_EPI_COMBINE_ADD = 1,  /* out_f32[slot / top_k] += row_weight[slot] * acc (top-k combine) */
  MOE_EPI_SCATTER_ROWS = 2  /* out[slot] = acc (unpermute; expert-parallel return path) */
} moe_epilogue_t;

/* Library version (major * 10000 + minor * 100 + patch). */
MOE_API int moe_version(void);
/* Message of the last failing call on this host thread ("" if none). */
MOE_API const char* moe_last_error(void);
/* Copies the device error flag (0 = none, else a code identifying the stalled
 * pipeline role: 1 TMA producer, 2 MMA issuer, 3 epilogue, 4 drain,
 * 6 self-test, 7 cross-CTA wait of the one-launch decode kernel) into
 * *host_code and clears it (after any error it also resets that kernel's
 * launch counter).
 * Synchronises `stream`. */
MOE_API int moe_get_device_error(int* host_code, void* stream);
/* Self-test of the bounded waits: one CTA waits on an mbarrier that nothing
 * completes; the wait gives up after timeout_ns (at most 2 s), the kernel
 * latches device error 6 and returns, and the context stays usable. */
MOE_API int moe_selftest_wait_timeout(uint64_t timeout_ns, void* stream);

/* Process-wide tuning options (moe_set_option / moe_get_option). */
typedef enum {
  MOE_OPT_GEMM_CTA_PAIR = 1 /* 1: grouped GEMMs run one tcgen05 MMA across a pair of CTAs on neighbouring
                               SMs (cta_group::2, 256-row tiles); 0: one CTA per 128-row tile; 2 (default):
                               pairs when the experts average at least 4 M tiles of 128 rows */,
  MOE_OPT_GEMM_BAND = 2     /* M tiles per band of the GEMMs' expert-major tile order (default 16): each
                               expert's tiles run in bands of this many M tiles, every band swept over
                               all N tiles, so CTAs running together share weight tiles in L2 */,
  MOE_OPT_GEMM_STREAM_K = 3 /* 1: the down GEMM with the combine epilogue (MOE_EPI_COMBINE_ADD, additive)
                               runs its full waves as whole tiles and splits the partial last wave's
                               (tile, K block) work evenly over the grid, adding partial sums;
                               0 (default): whole tiles only */,
  MOE_OPT_GEMM_HALF_UNITS = 4 /* CTA pairs only. 1 (default): an expert's odd last M tile runs as one
                               M=128 pair MMA, 64 of its rows on each CTA; 0: as an M=256 pair MMA
                               whose second CTA's rows are idle */,
  MOE_OPT_PDL = 5,            /* 1 (default): kernels are launched with programmatic dependent launch,
                               so each one's launch and prologue overlap the kernel before it in the
                               stream (every kernel first waits for its predecessors' results); 0: off */
  MOE_OPT_KERNEL_CLOCKS = 6,  /* 1: the grouped GEMM kernels time every launch on the device (read with
                               moe_kernel_clocks); launches are captured with the setting in force when
                               they are issued, so set it before capturing a CUDA graph. 0 (default): off */
  MOE_OPT_GEMM_SWAP_AB = 7    /* operand roles of the grouped GEMMs. 2 (default): the all-in-one entry points
                               swap them in the gate_up GEMM when the routed rows average at most 64 per
                               expert that receives any (decode), and in the down GEMM as well for at most
                               32 routed slots: the 128 weight rows of an output-feature tile are the MMA's M
                               operand and the expert's token rows (rounded up to 16) its N operand, with
                               the K dimension split over more CTAs when a launch has few work items; the
                               stand-alone GEMM entry points keep rows as M. 1: always swap (stand-alone
                               GEMMs included, without K splits). 0: never */,
  MOE_OPT_GEMM_BAND_DOWN = 8, /* the down GEMM's band of M tiles (MOE_OPT_GEMM_BAND); 0 (default): the same
                               band as the gate_up GEMM */
  MOE_OPT_DECODE_FUSED = 9    /* 1 (default): moe_fused_experts (and moe_fused_experts_from_logits, with its
                               router, up to 256 experts) runs a batch of at most 16 tokens and 128 routed
                               slots (bf16/fp16, no int8) as one persistent kernel — routing, gate_up GEMM +
                               SwiGLU, down GEMM + combine and output conversion as phases whose CTAs
                               hand results on through counters. Its launch counter lives in the library's
                               device memory, so two such calls must not run concurrently on one GPU
                               (different streams); callers that overlap MoE calls on several streams set 0.
                               With 1 a batch whose gate_up work is split along K runs as clusters of the
                               split CTAs, which add their partial sums through distributed shared memory
                               (when every cluster of the grid can be resident at once); 2: the same kernel
                               without clusters, partial sums through global memory */
} moe_option_t;
MOE_API int moe_set_option(int option, int value);
/* Current value of an option, or -1 for an unknown option. */
MOE_API int moe_get_option(int option);

/* Number of CUDA kernels this library has launched in this process
 * (monotonic, all threads). */
MOE_API int64_t moe_launch_count(void);

/* Device-side kernel clocks (MOE_OPT_KERNEL_CLOCKS): for each kernel class,
 * the summed busy time of its launches on the current device — from the
 * first CTA past its wait on the preceding kernels to the last CTA's end, so
 * a launch's prologue overlapped with its predecessor is not counted — and
 * the number of launches. Classes: MOE_CLOCK_GATE_UP (gate_up GEMM +
 * SwiGLU), MOE_CLOCK_DOWN (down GEMM + its epilogue). Copies the first n
 * classes into total_ns[] / launches[] (host arrays), clears them if reset
 * != 0, and synchronises `stream`. */
typedef enum { MOE_CLOCK_GATE_UP = 0, MOE_CLOCK_DOWN = 1, MOE_NUM_CLOCKS = 2 } moe_clock_t;
MOE_API int moe_kernel_clocks(uint64_t* total_ns, uint64_t* launches, int n, int reset, void* stream);

/* Stage boundaries at which the all-in-one entry points record profiling
 * events (moe_set_stage_events). */
typedef enum {
  MOE_STAGE_ENTRY = 0,
  MOE_STAGE_ROUTED = 1,   /* tile schedule / align done */
  MOE_STAGE_GATHERED = 2, /* permuting gather (+ int8 quant) done */
  MOE_STAGE_GEMM1 = 3,    /* gate_up GEMM + SwiGLU done */
  MOE_STAGE_PRE_GEMM2 = 4,/* int8 quant of h + output clear done */
  MOE_STAGE_GEMM2 = 5,    /* down GEMM + combine done */
  MOE_STAGE_DONE = 6,     /* output conversion done */
  MOE_NUM_STAGES = 7
} moe_stage_t;

/* Profiling hook (this host thread only): while `events` is non-NULL,
 * moe_fused_mlp and moe_fused_experts record events[i] (cudaEvent_t) on their
 * stream at stage boundary i < num_events. Pass NULL to disable. */
MOE_API int moe_set_stage_events(void* const* events, int num_events);

/* --------------------------------------------------------------------------
 * Tile schedule — replaces build_tile_schedule (fused_moe_mlp_triton.py:91-119).
 * For grid = ceil(num_tokens / block_m) + num_experts tiles (the reference's
 * static upper bound) writes, per tile i:
 *   tile_expert[i]    = searchsorted(cumsum(ceil(gs / block_m)), i, right=True),
 *                       clamped to num_experts - 1
 *   tile_row_start[i] = offsets[e] + (i - tiles_cumsum[e]) * block_m (0 if invalid)
 *   tile_row_count[i] = clamp(offsets[e + 1] - row_start, 0, block_m) (0 if invalid)
 * as int64, bit-identical to the reference. group_sizes is int32 or int64.
 * `tile_table` (optional, may be NULL) receives the compact int32 table the
 * GEMM entry points consume; its size is moe_tile_table_ints(E, grid).
 * -------------------------------------------------------------------------- */
MOE_API int64_t moe_tile_grid(int64_t num_tokens, int num_experts, int block_m);
MOE_API int64_t moe_tile_table_ints(int num_experts, int64_t max_tiles);
MOE_API int moe_tile_schedule(const void* group_sizes, int gs_dtype, int num_experts, int64_t num_tokens, int block_m,
                      int64_t* tile_expert, int64_t* tile_row_start, int64_t* tile_row_count,
                      int32_t* tile_table, void* stream);

/* --------------------------------------------------------------------------
 * Router (no reference counterpart: the reference's callers route with an
 * external op). logits [T, E] (fp32/bf16/fp16) -> topk_ids [T, k] int32 and
 * topk_weights [T, k] fp32. The k largest logits win, in descending order,
 * ties to the lower expert id (softmax and sigmoid are monotonic, so these
 * are the top-k scores). Weights: softmax: exp(l - max) / sum over all
 * experts, or over the k chosen when renormalize != 0; sigmoid:
 * 1 / (1 + exp(-l)), divided by the sum over the k chosen when renormalize.
 * E <= 1024, k <= min(E, 32).
 * -------------------------------------------------------------------------- */
typedef enum { MOE_SCORE_SOFTMAX = 0, MOE_SCORE_SIGMOID = 1 } moe_scoring_t;
MOE_API int moe_route_topk(const void* logits, int dtype, int64_t num_tokens, int num_experts, int top_k,
                           int scoring, int renormalize, int32_t* topk_ids, float* topk_weights, void* stream);

/* --------------------------------------------------------------------------
 * Routing align (no reference counterpart; upstream of fused_moe_mlp, the
 * contract of "tokens grouped contiguously by expert, expert 0 first",
 * independent_test.py:24-31). Stable counting sort of the num_tokens*top_k
 * slots (slot = t * top_k + j) by expert id, each expert's segment padded to
 * a multiple of block_m rows:
 *   sorted_slots[p]  slot id at padded row p, or -1 for padding rows
 *   slot_pos[slot]   padded row of the slot, -1 if its id is outside [0, E)
 *   group_sizes[e]   number of slots routed to expert e (int32)
 *   padded_offsets[e] first padded row of expert e; [E] = total padded rows
 *   tile_table       compact schedule consumed by the GEMMs
 * Ids outside [0, num_experts) are dropped (counted in tile_table[2]).
 * sorted_slots needs moe_align_capacity() entries: num_slots plus block_m - 1
 * padding rows for each expert that can hold a slot (at most
 * min(num_experts, num_slots)), rounded up to whole tiles of block_m rows.
 * -------------------------------------------------------------------------- */
MOE_API int64_t moe_align_capacity(int64_t num_slots, int num_experts, int block_m);
MOE_API size_t moe_align_workspace_size(int64_t num_tokens, int top_k, int num_experts, int block_m);
MOE_API int moe_align(const int32_t* topk_ids, int64_t num_tokens, int top_k, int num_experts, int block_m,
              int32_t* sorted_slots, int32_t* slot_pos, int32_t* group_sizes, int32_t* padded_offsets,
              int32_t* tile_table, void* workspace, size_t workspace_bytes, void* stream);

/* moe_align without a workspace argument, for callers that cannot allocate
 * device memory at all — for example a plugin that a host engine hands only
 * its input and output buffers, or a serving process whose memory pool is
 * fully reserved at start-up so no cudaMalloc may happen afterwards. It has
 * no counterpart in the reference. Outputs and their meaning are exactly
 * those of moe_align; it allocates nothing and calls no cudaMalloc/cudaFree.
 * Batches of at most 16384 slots over at most 1024 experts run the one-CTA
 * align, which needs no scratch. Larger ones keep their scratch in a
 * file-scope device array of MOE_ALIGN_STATIC_SCRATCH_BYTES (1 MiB) that
 * every GPU which loads this library holds until the process exits; requests
 * whose scratch (moe_align_workspace_size) exceeds it fail with
 * MOE_ERR_INVALID_ARG. Example, top-8 over 256 experts: 8192 tokens need
 * 0.50 MiB and fit, the limit is 16288 tokens, and 16384 tokens (1.005 MiB)
 * are rejected. The first call on each device that uses the array looks up
 * its device address with that device current (again after the device's
 * context is recreated, e.g. by cudaDeviceReset); make that first call before
 * any stream capture. All calls share the one array and it keeps the last
 * call's contents: calls that overlap on the GPU (other streams, other host
 * threads) race with each other and must be serialised by the caller. */
#define MOE_ALIGN_STATIC_SCRATCH_BYTES (1u << 20)
MOE_API int moe_align_static(const int32_t* topk_ids, int64_t num_tokens, int top_k, int num_experts, int block_m,
                             int32_t* sorted_slots, int32_t* slot_pos, int32_t* group_sizes,
                             int32_t* padded_offsets, int32_t* tile_table, void* stream);

/* --------------------------------------------------------------------------
 * Row gather and per-token int8 quant (no reference counterpart).
 * moe_gather_rows: dst[p] = src[sorted_slots[p] / top_k] for p < rows
 * (zero rows where sorted_slots[p] < 0). If dst_dtype == MOE_I8 the row is
 * quantised on the fly: s = absmax / 127, q = clamp(rint(x * (127 / absmax)),
 * -127, 127) (fp32, round-half-even; s = 0 and q = 0 for an all-zero row), s written to
 * dst_scale[p]. `rows_dev` (optional) points at a device int bounding the
 * rows processed (e.g. tile_table + 1); `rows` is the static upper bound.
 * moe_quant_rows: the same quantisation applied row-by-row in place order.
 * -------------------------------------------------------------------------- */
MOE_API int moe_gather_rows(const void* src, int src_dtype, int64_t cols, const int32_t* sorted_slots, int top_k,
                    int64_t rows, const int32_t* rows_dev, void* dst, int dst_dtype, float* dst_scale,
                    void* stream);
MOE_API int moe_quant_rows(const void* src, int src_dtype, int64_t rows, int64_t cols, const int32_t* rows_dev,
                   int8_t* dst, float* dst_scale, void* stream);

/* --------------------------------------------------------------------------
 * Grouped GEMMs (tcgen05 / TMEM, TMA-fed, persistent, warp-specialised).
 * Replaces _grouped_gemm1_swiglu_kernel (partially_fused_moe_mlp_triton.py:59-114)
 * and the GEMM1 half of _fused_moe_mlp_kernel (fused_moe_mlp_triton.py:35-66):
 *   h[r, n] = silu(g) * u,  g = a[r] . w13[e, n],  u = a[r] . w13[e, I + n]
 * with fp32 (int32 for int8) accumulation; w8a8 dequant (a_scale[r] *
 * w13_scale[e, n]) is applied to g and u before the SwiGLU. h is written in
 * h_dtype (the reference's weight dtype; bf16 for int8 inputs).
 * a: [a_rows, H]; w13: [E, 2I, H]; h: [a_rows, I]. dtypes: BF16, F16, F32
 * (tf32 tensor cores), I8 (a and w13 both int8, scales required). Up to
 * 1024 experts.
 * -------------------------------------------------------------------------- */
MOE_API int moe_gemm1_swiglu(const void* a, int dtype, int64_t a_rows, int64_t hidden, const void* w13,
                     int num_experts, int64_t inter, const float* a_scale, const float* w13_scale,
                     const int32_t* tile_table, int64_t max_tiles, void* h, int h_dtype, void* stream);

/* Replaces _grouped_gemm2_kernel (partially_fused_moe_mlp_triton.py:116-162)
 * and the GEMM2 half of _fused_moe_mlp_kernel (fused_moe_mlp_triton.py:68-88):
 *   acc[r, c] = h[r] . w2[e, c]   (w2: [E, H, I], h: [h_rows, I])
 * dequantised by h_scale[r] * w2_scale[e, c] for int8, then per `epilogue`:
 *   MOE_EPI_STORE_ROWS   out[r, c] = acc                       (out_dtype)
 *   MOE_EPI_COMBINE_ADD  out[row_map[r] / top_k, c] += row_weight[row_map[r]] * acc
 *                        (out is fp32, atomically accumulated; rows with
 *                        row_map < 0 skipped) — the top-k weighted unpermute
 *                        and combine of the MoE layer
 *   MOE_EPI_SCATTER_ROWS out[row_map[r], c] = acc (x row_weight[row_map[r]] if
 *                        row_weight != NULL), out_dtype
 * -------------------------------------------------------------------------- */
MOE_API int moe_gemm2(const void* h, int dtype, int64_t h_rows, int64_t inter, const void* w2, int num_experts,
              int64_t hidden, const float* h_scale, const float* w2_scale, const int32_t* tile_table,
              int64_t max_tiles, int epilogue, const int32_t* row_map, const float* row_weight, int top_k,
              void* out, int out_dtype, int64_t out_rows, void* stream);

/* y[t, c] = sum_j topk_weights[t, j] * o[slot_pos[t*k + j], c] (fp32 sum,
 * skipped where slot_pos < 0), written in y_dtype. Deterministic combine used
 * by the expert-parallel path. */
MOE_API int moe_combine_rows(const void* o, int o_dtype, int64_t hidden, const int32_t* slot_pos,
                     const float* topk_weights, int64_t num_tokens, int top_k, void* y, int y_dtype,
                     void* stream);

/* dst[i] = (dst_dtype) src_f32[i] for i < n. */
MOE_API int moe_convert_f32(const float* src, int64_t n, void* dst, int dst_dtype, void* stream);

/* --------------------------------------------------------------------------
 * All-in-one entry points.
 *
 * moe_fused_mlp — drop-in for fused_moe_mlp(x, w13, w2, group_sizes)
 * (fused_moe_mlp_triton.py:121-160; call site unquant_diff.txt:13-18): x is
 * [num_tokens, H] already grouped by expert, group_sizes [E] (int32/int64)
 * counts, out [num_tokens, H] in x's dtype (rows no group covers are zero).
 * dtype in {BF16, F16, F32}; block_m must be 128.
 *
 * moe_fused_experts — the top-k form fused_moe_mlp(hidden_states, w13, w2,
 * topk_weights, topk_ids, [scales]): align -> gather (+int8 quant) -> GEMM1 +
 * SwiGLU -> (int8 quant of h) -> GEMM2 + weighted combine -> y [T, H] in
 * x_dtype. The combine is fused into GEMM2's epilogue (fp32 atomics) while
 * the T x H fp32 accumulator fits in L2 (<= 80 MiB); larger outputs store
 * GEMM2 rows and sum them per token with moe_combine_rows. w_dtype == MOE_I8 selects w8a8 with per-output-channel weight
 * scales w13_scale [E, 2I] and w2_scale [E, H] (fp32) and dynamic per-token
 * activation scales; otherwise w_dtype must equal x_dtype.
 * -------------------------------------------------------------------------- */
MOE_API size_t moe_fused_mlp_workspace_size(int64_t num_tokens, int64_t hidden, int64_t inter, int num_experts,
                                    int dtype, int block_m);
MOE_API int moe_fused_mlp(const void* x, int dtype, int64_t num_tokens, int64_t hidden, const void* w13,
                  const void* w2, int num_experts, int64_t inter, const void* group_sizes, int gs_dtype,
                  int block_m, void* out, void* workspace, size_t workspace_bytes, void* stream);

MOE_API size_t moe_fused_experts_workspace_size(int64_t num_tokens, int64_t hidden, int64_t inter, int num_experts,
                                        int top_k, int x_dtype, int w_dtype);
MOE_API int moe_fused_experts(const void* x, int x_dtype, int64_t num_tokens, int64_t hidden, const void* w13,
                      const void* w2, int w_dtype, int num_experts, int64_t inter, const float* topk_weights,
                      const int32_t* topk_ids, int top_k, const float* w13_scale, const float* w2_scale,
                      void* y, void* workspace, size_t workspace_bytes, void* stream);

/* moe_fused_experts_from_logits — routing and the layer in one call (no
 * reference counterpart: the reference's callers route with an external op).
 * The router of moe_route_topk (same selection, tie rule and weights) turns
 * router_logits [T, E] (fp32/bf16/fp16) into topk_ids [T, k] and topk_weights
 * [T, k], both written as outputs, and moe_fused_experts runs on them. A batch
 * that takes the one-launch decode kernel (MOE_OPT_DECODE_FUSED) with
 * E <= 256 routes inside that kernel's first phase, so the whole layer,
 * routing included, is one launch; other batches launch the router first.
 * Workspace: moe_fused_experts_workspace_size with the same sizes. */
MOE_API int moe_fused_experts_from_logits(const void* x, int x_dtype, int64_t num_tokens, int64_t hidden,
                                          const void* w13, const void* w2, int w_dtype, int num_experts,
                                          int64_t inter, const void* router_logits, int logits_dtype, int top_k,
                                          int scoring, int renormalize, int32_t* topk_ids, float* topk_weights,
                                          const float* w13_scale, const float* w2_scale, void* y, void* workspace,
                                          size_t workspace_bytes, void* stream);

/* moe_fused_expert_rows — the expert MLP applied row by row, with no routing
 * weights and no combine: out[r] = MLP_{expert_ids[r]}(x[r]) for r < rows,
 * in x_dtype (rows whose id is outside [0, E) are left unwritten). This is
 * the local pass of expert parallelism, where each received row carries one
 * local expert id and its result travels back unweighted. No reference
 * counterpart. */
MOE_API size_t moe_fused_expert_rows_workspace_size(int64_t rows, int64_t hidden, int64_t inter, int num_experts,
                                                    int x_dtype, int w_dtype);
MOE_API int moe_fused_expert_rows(const void* x, int x_dtype, int64_t rows, int64_t hidden, const void* w13,
                                  const void* w2, int w_dtype, int num_experts, int64_t inter,
                                  const int32_t* expert_ids, const float* w13_scale, const float* w2_scale,
                                  void* out, void* workspace, size_t workspace_bytes, void* stream);

/* --------------------------------------------------------------------------
 * Expert parallelism over NVLink peer memory (no reference counterpart: the
 * reference has no distributed code). Rank r of W owns experts
 * [r*EL, (r+1)*EL). Each rank allocates once (moe_ipc_malloc) a receive
 * buffer of recv_cap rows laid out as the padded, expert-sorted input of its
 * local experts, a row-tag array (int32 per row) and a return buffer, and
 * opens its peers' buffers (moe_ipc_open). Per forward:
 *   moe_align(block_m = 1) of the local top-k ids; all-gather of the
 *   group sizes into counts_all [W, E] (int32);
 *   moe_ep_plan: dest_base[e] = first row of this rank's expert-e rows in the
 *     owner's buffer; this rank's tile table over its local experts; tag -1
 *     on its own padding rows; ret_pos[s] = s for routed slots, else -1;
 *   moe_ep_dispatch: row of every routed slot stored into the owner's buffer
 *     (peer stores; int8-quantised when recv_dtype is MOE_I8) with tag
 *     (rank << 24) | slot;
 *   barrier across ranks;
 *   moe_ep_expert_pass: local gate_up GEMM + SwiGLU, down GEMM whose
 *     epilogue stores row r to peer_ret[tag >> 24] at row tag & 0xFFFFFF;
 *   barrier; moe_combine_rows(return buffer, ret_pos, topk_weights).
 * peer_* arguments are device arrays of W device pointers.
 * -------------------------------------------------------------------------- */
#define MOE_IPC_HANDLE_BYTES 64
MOE_API int moe_ipc_malloc(size_t bytes, void** ptr, void* handle);
MOE_API int moe_ipc_open(const void* handle, void** ptr);
MOE_API int moe_ipc_close(void* ptr);
MOE_API int moe_ipc_free(void* ptr);
MOE_API int moe_ep_plan(const int32_t* counts_all, int world, int rank, int num_experts, const int32_t* slot_pos,
                        int64_t num_slots, int32_t* dest_base, int32_t* tile_table, int64_t max_tiles,
                        int32_t* recv_meta, int64_t recv_cap, int32_t* ret_pos, void* stream);
MOE_API int moe_ep_dispatch(const void* x, int x_dtype, int64_t hidden, int top_k, const int32_t* topk_ids,
                            const int32_t* sorted_slots, const int32_t* seg_start, const int32_t* dest_base,
                            const int32_t* n_valid_dev, int64_t max_rows, int world, int rank,
                            int experts_per_rank, int64_t recv_cap, void* const* peer_x, int recv_dtype,
                            float* const* peer_scale, int32_t* const* peer_meta, int* err, void* stream);
MOE_API size_t moe_ep_expert_pass_workspace_size(int64_t recv_cap, int64_t inter, int x_dtype);
MOE_API int moe_ep_expert_pass(const void* recv_x, int x_dtype, const float* recv_scale, int64_t recv_cap,
                               int64_t hidden, const void* w13, const void* w2, int experts_per_rank,
                               int64_t inter, const float* w13_scale, const float* w2_scale,
                               const int32_t* tile_table, const int32_t* recv_meta, void* const* peer_ret,
                               int world, int64_t ret_rows, int out_dtype, void* workspace,
                               size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H_ */
