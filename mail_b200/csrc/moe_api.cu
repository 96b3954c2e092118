// All-in-one entry points and error reporting of the C ABI.
//
//   moe_fused_mlp      drop-in for fused_moe_mlp(x, w13, w2, group_sizes)
//                      (fused_moe_mlp_triton.py:121-160): tile schedule ->
//                      GEMM1 + SwiGLU -> GEMM2 with a row-store epilogue.
//   moe_fused_experts  the top-k form: align -> gather (+ int8 quant) ->
//                      GEMM1 + SwiGLU -> (int8 quant of h) -> GEMM2 with the
//                      weighted scatter-add combine -> output dtype.
#include <atomic>
#include <string>

#include "common.cuh"

namespace moe {

namespace {
thread_local std::string g_last_error;
std::atomic<int64_t> g_launches{0};
thread_local void* const* g_stage_events = nullptr;
thread_local int g_num_stage_events = 0;

}  // namespace

int record_stage(int stage, cudaStream_t st) {
  if (g_stage_events && stage < g_num_stage_events && g_stage_events[stage]) {
    // under stream capture an event record becomes a graph node only with
    // cudaEventRecordExternal (a plain record would only order the capture)
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    MOE_CUDA_TRY(cudaStreamIsCapturing(st, &cs));
    const unsigned flags = cs == cudaStreamCaptureStatusActive ? cudaEventRecordExternal : cudaEventRecordDefault;
    MOE_CUDA_TRY(cudaEventRecordWithFlags(static_cast<cudaEvent_t>(g_stage_events[stage]), st, flags));
  }
  return MOE_OK;
}

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

namespace {

// Workspace carve-out helper: each region 256-byte aligned.
struct Carver {
  size_t off = 0;
  size_t take(size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  }
};

struct FusedMlpWs {
  int64_t grid;
  size_t table, h, bytes;
};
FusedMlpWs fused_mlp_ws(int64_t T, int64_t I, int E, int dtype, int block_m) {
  FusedMlpWs w;
  w.grid = ceil_div(T, block_m) + E;
  Carver c;
  w.table = c.take(TileTable::ints(E, w.grid) * sizeof(int32_t));
  w.h = c.take((size_t)T * I * dtype_size(dtype));
  w.bytes = c.off;
  return w;
}

// Output handling of the top-k expert pass.
enum class ExpertsOut {
  kCombineAtomic,  // GEMM2 epilogue scatter-adds w * row into an fp32 [T, H] accumulator
  kCombineRows,    // GEMM2 stores rows [cap, H]; moe_combine_rows sums the k rows per token
  kScatterRows     // k = 1, unit weight: GEMM2 writes row r of the output directly
};

// The fused atomic combine pays off while its fp32 accumulator stays
// resident in the 126 MB L2 next to the other traffic; above this size the
// read-modify-writes reach HBM and a row store + separate combine is cheaper.
constexpr size_t kAtomicCombineMaxBytes = size_t(80) << 20;

// Largest batch whose output conversion runs inside the down GEMM.
constexpr int64_t kFusedConvertMaxTokens = 32;

ExpertsOut combine_mode(int64_t T, int64_t H) {
  return (size_t)T * H * sizeof(float) <= kAtomicCombineMaxBytes ? ExpertsOut::kCombineAtomic
                                                                  : ExpertsOut::kCombineRows;
}

struct FusedExpertsWs {
  int64_t S, cap, max_tiles;
  size_t align_bytes;
  GemmPlan plan;
  bool small;         // decode-sized: one prep launch, output conversion fused into the down GEMM
  bool fused_convert;
  size_t align, sorted, slot_pos, gs, poff, table, xp, xs, h, hq, hs, y32, o, partial, counters, conv_cnt, kvalid,
      zero_end, bytes;
};
FusedExpertsWs fused_experts_ws(int64_t T, int64_t H, int64_t I, int E, int k, int x_dtype, int w_dtype,
                                ExpertsOut mode) {
  FusedExpertsWs w;
  w.S = T * k;
  w.cap = moe_align_capacity(w.S, E, kBlockM);
  w.max_tiles = w.cap / kBlockM;
  w.align_bytes = moe_align_workspace_size(T, k, E, kBlockM);
  const bool q = (w_dtype == MOE_I8);
  const int h_dtype = (x_dtype == MOE_F32) ? MOE_F32 : (q ? MOE_BF16 : x_dtype);
  Carver c;
  w.align = c.take(w.align_bytes);
  w.sorted = c.take(w.cap * sizeof(int32_t));
  w.slot_pos = c.take(w.S * sizeof(int32_t));
  w.gs = c.take(E * sizeof(int32_t));
  w.poff = c.take((E + 1) * sizeof(int32_t));
  w.table = c.take(TileTable::ints(E, w.max_tiles) * sizeof(int32_t));
  w.xp = c.take((size_t)w.cap * H * (q ? 1 : dtype_size(x_dtype)));
  w.xs = c.take(q ? w.cap * sizeof(float) : 0);
  w.h = c.take((size_t)w.cap * I * dtype_size(h_dtype));
  w.hq = c.take(q ? (size_t)w.cap * I : 0);
  w.hs = c.take(q ? w.cap * sizeof(float) : 0);
  const bool atomic_acc = mode == ExpertsOut::kCombineAtomic && x_dtype != MOE_F32;
  w.y32 = c.take(atomic_acc ? (size_t)T * H * sizeof(float) : 0);
  w.o = c.take(mode == ExpertsOut::kCombineRows ? (size_t)w.cap * H * dtype_size(x_dtype) : 0);
  w.plan = gemm_plan(w.S, E, w.max_tiles, H, I, q ? MOE_I8 : x_dtype, mode == ExpertsOut::kCombineAtomic);
  w.small = mode == ExpertsOut::kCombineAtomic && prep_small_fits(w.S, E);
  // fused conversion: saves the convert launch where it is a sizeable share of
  // the step (a few tokens); per-token completion counts cost more above that
  w.fused_convert = w.small && w.plan.swap2 && x_dtype != MOE_F32 && T <= kFusedConvertMaxTokens;
  w.partial = c.take(w.plan.partial_bytes);
  // zero-filled together by the prep launch: split-K counts, conversion counts
  w.counters = c.take(w.plan.counter_bytes);
  w.conv_cnt = c.take(w.fused_convert ? (size_t)T * ceil_div(H, 128) * 4 * sizeof(int32_t) : 0);
  w.zero_end = c.off;
  w.kvalid = c.take(w.fused_convert ? (size_t)T * sizeof(int32_t) : 0);
  w.bytes = c.off;
  return w;
}

struct ExpertsArgs {
  const void* x;
  int x_dtype;
  int64_t T, H;
  const void* w13;
  const void* w2;
  int w_dtype, E;
  int64_t I;
  const float* topk_weights;  // NULL for kScatterRows
  const int32_t* topk_ids;
  int k;
  const float* w13_scale;
  const float* w2_scale;
  void* y;
  void* workspace;
  size_t workspace_bytes;
  void* stream;
  ExpertsOut mode;
  const char* name;
};

int check_experts(const ExpertsArgs& a) {
  MOE_CHECK_ARG(a.x_dtype == MOE_BF16 || a.x_dtype == MOE_F16 || a.x_dtype == MOE_F32,
                "%s: x dtype must be bf16, fp16 or fp32", a.name);
  MOE_CHECK_ARG(a.w_dtype == a.x_dtype || a.w_dtype == MOE_I8,
                "%s: weights must share x's dtype or be int8 (w8a8)", a.name);
  MOE_CHECK_ARG(!(a.w_dtype == MOE_I8 && a.x_dtype == MOE_F32), "%s: w8a8 takes bf16/fp16 activations", a.name);
  if (a.w_dtype == MOE_I8) MOE_CHECK_ARG(a.w13_scale && a.w2_scale, "%s: int8 weights need scales", a.name);
  MOE_CHECK_ARG(a.T >= 0 && a.H > 0 && a.I > 0 && a.E > 0 && a.k > 0, "%s: bad sizes", a.name);
  MOE_CHECK_ARG(a.T == 0 || a.y != nullptr, "%s: output is NULL", a.name);  // empty batch: nothing to write
  return MOE_OK;
}

bool one_launch(const ExpertsArgs& a) {
  return a.mode == ExpertsOut::kCombineAtomic && decode_fused_fits(a.T, a.k, a.E, a.H, a.I, a.x_dtype, a.w_dtype);
}

// align -> gather (+int8 quant) -> GEMM1 + SwiGLU -> (int8 quant of h) ->
// GEMM2 with the output handling of a.mode; a decode-sized batch as one launch.
int run_experts(const ExpertsArgs& a) {
  if (a.T == 0) return MOE_OK;
  MOE_CHECK_ARG(a.x && a.w13 && a.w2 && a.topk_ids && (a.topk_weights || a.mode == ExpertsOut::kScatterRows),
                "%s: NULL input", a.name);
  if (one_launch(a)) {
    cudaStream_t st = as_stream(a.stream);
    MOE_TRY(record_stage(MOE_STAGE_ENTRY, st));
    MOE_TRY(decode_fused(a.x, a.x_dtype, a.T, a.H, a.w13, a.w2, a.E, a.I, a.topk_weights, a.topk_ids, a.k, a.y,
                         a.workspace, a.workspace_bytes, st));
    for (int s = MOE_STAGE_ROUTED; s <= MOE_STAGE_DONE; ++s) MOE_TRY(record_stage(s, st));
    return MOE_OK;
  }
  const FusedExpertsWs w = fused_experts_ws(a.T, a.H, a.I, a.E, a.k, a.x_dtype, a.w_dtype, a.mode);
  if (a.workspace_bytes < w.bytes || !a.workspace)
    return set_error(MOE_ERR_WORKSPACE, "%s: workspace %zu < %zu bytes", a.name, a.workspace_bytes, w.bytes);
  char* ws = static_cast<char*>(a.workspace);
  int32_t* sorted = reinterpret_cast<int32_t*>(ws + w.sorted);
  int32_t* slot_pos = reinterpret_cast<int32_t*>(ws + w.slot_pos);
  int32_t* gs = reinterpret_cast<int32_t*>(ws + w.gs);
  int32_t* poff = reinterpret_cast<int32_t*>(ws + w.poff);
  int32_t* table = reinterpret_cast<int32_t*>(ws + w.table);
  const bool q = (a.w_dtype == MOE_I8);
  const int h_dtype = (a.x_dtype == MOE_F32) ? MOE_F32 : (q ? MOE_BF16 : a.x_dtype);
  void* stream = a.stream;
  cudaStream_t st = as_stream(stream);

  MOE_TRY(record_stage(MOE_STAGE_ENTRY, st));
  const int32_t* rows_dev = table + 1;  // padded rows in use
  void* xp = ws + w.xp;
  float* xs = q ? reinterpret_cast<float*>(ws + w.xs) : nullptr;
  void* h = ws + w.h;
  int32_t* counters = w.plan.counter_bytes ? reinterpret_cast<int32_t*>(ws + w.counters) : nullptr;
  float* acc = nullptr;
  if (a.mode == ExpertsOut::kCombineAtomic)
    acc = (a.x_dtype == MOE_F32) ? static_cast<float*>(a.y) : reinterpret_cast<float*>(ws + w.y32);
  // decode-sized batches: align, gather (+ quant) and the zero fills in one launch
  const bool small = w.small;
  int32_t* kvalid = w.fused_convert ? reinterpret_cast<int32_t*>(ws + w.kvalid) : nullptr;
  if (small) {
    MOE_TRY(prep_small(a.topk_ids, a.T, a.k, a.E, kBlockM, a.x, a.x_dtype, a.H, xp, q, xs, sorted, slot_pos, gs,
                       poff, table, acc, (size_t)a.T * a.H * sizeof(float), ws + w.counters,
                       w.zero_end - w.counters, kvalid, a.y, st));
    MOE_TRY(record_stage(MOE_STAGE_ROUTED, st));
    MOE_TRY(record_stage(MOE_STAGE_GATHERED, st));
  } else {
    MOE_TRY(moe_align(a.topk_ids, a.T, a.k, a.E, kBlockM, sorted, slot_pos, gs, poff, table, ws + w.align,
                      w.align_bytes, stream));
    MOE_TRY(record_stage(MOE_STAGE_ROUTED, st));
    // padding rows are left as they are: the GEMMs never store their results.
    // Token order: each activation row is read (and quantised) once and
    // stored to its k padded rows
    if (scatter_rows_fits(a.H))
      MOE_TRY(scatter_rows(a.x, a.x_dtype, a.H, slot_pos, a.k, a.T, xp, q ? MOE_I8 : a.x_dtype, xs, st));
    else
      MOE_TRY(gather_rows(a.x, a.x_dtype, a.H, sorted, a.k, w.cap, rows_dev, xp, q ? MOE_I8 : a.x_dtype, xs, false,
                          stream));
    MOE_TRY(record_stage(MOE_STAGE_GATHERED, st));
    if (counters) MOE_TRY(zero_fill(counters, w.plan.counter_bytes, st));  // split-K counts start at zero
  }
  MOE_TRY(gemm1_swiglu_planned(xp, q ? MOE_I8 : a.x_dtype, w.cap, a.H, a.w13, a.E, a.I, xs, a.w13_scale, table,
                               w.max_tiles, h, h_dtype, &w.plan, ws + w.partial, counters, st));
  MOE_TRY(record_stage(MOE_STAGE_GEMM1, st));
  const void* a2 = h;
  float* hs = nullptr;
  if (q) {
    int8_t* hq = reinterpret_cast<int8_t*>(ws + w.hq);
    hs = reinterpret_cast<float*>(ws + w.hs);
    MOE_TRY(moe_quant_rows(h, h_dtype, w.cap, a.I, rows_dev, hq, hs, stream));
    a2 = hq;
  }
  const int g2_dtype = q ? MOE_I8 : h_dtype;
  if (a.mode == ExpertsOut::kCombineAtomic) {
    if (!small) MOE_TRY(zero_fill(acc, (size_t)a.T * a.H * sizeof(float), st));
    MOE_TRY(record_stage(MOE_STAGE_PRE_GEMM2, st));
    FusedConvert conv{a.y, a.x_dtype, reinterpret_cast<int32_t*>(ws + w.conv_cnt), kvalid};
    MOE_TRY(gemm2_planned(a2, g2_dtype, w.cap, a.I, a.w2, a.E, a.H, hs, a.w2_scale, table, w.max_tiles,
                          MOE_EPI_COMBINE_ADD, sorted, a.topk_weights, a.k, acc, MOE_F32, a.T, &w.plan, st,
                          w.fused_convert ? &conv : nullptr));
    MOE_TRY(record_stage(MOE_STAGE_GEMM2, st));
    if (a.x_dtype != MOE_F32 && !w.fused_convert) MOE_TRY(moe_convert_f32(acc, a.T * a.H, a.y, a.x_dtype, stream));
  } else if (a.mode == ExpertsOut::kCombineRows) {
    void* o = ws + w.o;
    MOE_TRY(record_stage(MOE_STAGE_PRE_GEMM2, st));
    MOE_TRY(gemm2_planned(a2, g2_dtype, w.cap, a.I, a.w2, a.E, a.H, hs, a.w2_scale, table, w.max_tiles,
                          MOE_EPI_STORE_ROWS, nullptr, nullptr, 1, o, a.x_dtype, w.cap, &w.plan, st));
    MOE_TRY(record_stage(MOE_STAGE_GEMM2, st));
    MOE_TRY(moe_combine_rows(o, a.x_dtype, a.H, slot_pos, a.topk_weights, a.T, a.k, a.y, a.x_dtype, stream));
  } else {
    MOE_TRY(record_stage(MOE_STAGE_PRE_GEMM2, st));
    MOE_TRY(gemm2_planned(a2, g2_dtype, w.cap, a.I, a.w2, a.E, a.H, hs, a.w2_scale, table, w.max_tiles,
                          MOE_EPI_SCATTER_ROWS, sorted, nullptr, 1, a.y, a.x_dtype, a.T, &w.plan, st));
    MOE_TRY(record_stage(MOE_STAGE_GEMM2, st));
  }
  MOE_TRY(record_stage(MOE_STAGE_DONE, st));
  return MOE_OK;
}

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" int moe_version(void) { return 100; }

extern "C" const char* moe_last_error(void) { return g_last_error.c_str(); }

extern "C" int64_t moe_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" int moe_set_stage_events(void* const* events, int num_events) {
  MOE_CHECK_ARG(events == nullptr || num_events >= 0, "moe_set_stage_events: bad count");
  g_stage_events = events;
  g_num_stage_events = events ? num_events : 0;
  return MOE_OK;
}

extern "C" size_t moe_fused_mlp_workspace_size(int64_t num_tokens, int64_t hidden, int64_t inter, int num_experts,
                                               int dtype, int block_m) {
  (void)hidden;
  if (num_tokens < 0 || inter <= 0 || num_experts <= 0 || block_m != kBlockM || dtype_size(dtype) == 0) return 0;
  return fused_mlp_ws(num_tokens, inter, num_experts, dtype, block_m).bytes;
}

extern "C" int moe_fused_mlp(const void* x, int dtype, int64_t num_tokens, int64_t hidden, const void* w13,
                             const void* w2, int num_experts, int64_t inter, const void* group_sizes, int gs_dtype,
                             int block_m, void* out, void* workspace, size_t workspace_bytes, void* stream) {
  MOE_CHECK_ARG(dtype == MOE_BF16 || dtype == MOE_F16 || dtype == MOE_F32,
                "moe_fused_mlp: dtype must be bf16, fp16 or fp32");
  MOE_CHECK_ARG(block_m == kBlockM, "moe_fused_mlp: block_m must be %d on sm_100a (got %d)", kBlockM, block_m);
  MOE_CHECK_ARG(num_tokens >= 0 && hidden > 0 && inter > 0 && num_experts > 0, "moe_fused_mlp: bad sizes");
  MOE_CHECK_ARG(num_tokens == 0 || out != nullptr, "moe_fused_mlp: out is NULL");
  if (num_tokens == 0) return MOE_OK;  // empty batch: empty output, as the reference returns
  const FusedMlpWs w = fused_mlp_ws(num_tokens, inter, num_experts, dtype, block_m);
  if (workspace_bytes < w.bytes || !workspace)
    return set_error(MOE_ERR_WORKSPACE, "moe_fused_mlp: workspace %zu < %zu bytes", workspace_bytes, w.bytes);
  char* ws = static_cast<char*>(workspace);
  int32_t* table = reinterpret_cast<int32_t*>(ws + w.table);
  void* h = ws + w.h;
  cudaStream_t st = as_stream(stream);
  MOE_TRY(record_stage(MOE_STAGE_ENTRY, st));
  MOE_TRY(moe_tile_schedule(group_sizes, gs_dtype, num_experts, num_tokens, block_m, nullptr, nullptr, nullptr,
                            table, stream));
  // the reference zero-initialises its output; rows no group covers stay 0
  MOE_TRY(zero_fill(out, (size_t)num_tokens * hidden * dtype_size(dtype), st));
  MOE_TRY(record_stage(MOE_STAGE_ROUTED, st));
  MOE_TRY(record_stage(MOE_STAGE_GATHERED, st));
  MOE_TRY(moe_gemm1_swiglu(x, dtype, num_tokens, hidden, w13, num_experts, inter, nullptr, nullptr, table, w.grid, h,
                           dtype, stream));
  MOE_TRY(record_stage(MOE_STAGE_GEMM1, st));
  MOE_TRY(record_stage(MOE_STAGE_PRE_GEMM2, st));
  MOE_TRY(moe_gemm2(h, dtype, num_tokens, inter, w2, num_experts, hidden, nullptr, nullptr, table, w.grid,
                    MOE_EPI_STORE_ROWS, nullptr, nullptr, 1, out, dtype, num_tokens, stream));
  MOE_TRY(record_stage(MOE_STAGE_GEMM2, st));
  MOE_TRY(record_stage(MOE_STAGE_DONE, st));
  return MOE_OK;
}

extern "C" size_t moe_fused_experts_workspace_size(int64_t num_tokens, int64_t hidden, int64_t inter,
                                                   int num_experts, int top_k, int x_dtype, int w_dtype) {
  if (num_tokens < 0 || hidden <= 0 || inter <= 0 || num_experts <= 0 || top_k <= 0) return 0;
  if (dtype_size(x_dtype) == 0 || dtype_size(w_dtype) == 0) return 0;
  const ExpertsOut mode = combine_mode(num_tokens, hidden);
  if (mode == ExpertsOut::kCombineAtomic &&
      decode_fused_fits(num_tokens, top_k, num_experts, hidden, inter, x_dtype, w_dtype))
    return decode_fused_workspace(num_tokens, top_k, num_experts, hidden, inter, x_dtype);
  return fused_experts_ws(num_tokens, hidden, inter, num_experts, top_k, x_dtype, w_dtype, mode).bytes;
}

extern "C" int moe_fused_experts(const void* x, int x_dtype, int64_t num_tokens, int64_t hidden, const void* w13,
                                 const void* w2, int w_dtype, int num_experts, int64_t inter,
                                 const float* topk_weights, const int32_t* topk_ids, int top_k,
                                 const float* w13_scale, const float* w2_scale, void* y, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  ExpertsArgs a{x, x_dtype, num_tokens, hidden, w13, w2, w_dtype, num_experts, inter, topk_weights, topk_ids,
                top_k, w13_scale, w2_scale, y, workspace, workspace_bytes, stream,
                combine_mode(num_tokens, hidden), "moe_fused_experts"};
  MOE_TRY(check_experts(a));
  return run_experts(a);
}

extern "C" int moe_fused_experts_from_logits(const void* x, int x_dtype, int64_t num_tokens, int64_t hidden,
                                             const void* w13, const void* w2, int w_dtype, int num_experts,
                                             int64_t inter, const void* router_logits, int logits_dtype, int top_k,
                                             int scoring, int renormalize, int32_t* topk_ids, float* topk_weights,
                                             const float* w13_scale, const float* w2_scale, void* y,
                                             void* workspace, size_t workspace_bytes, void* stream) {
  ExpertsArgs a{x, x_dtype, num_tokens, hidden, w13, w2, w_dtype, num_experts, inter, topk_weights, topk_ids,
                top_k, w13_scale, w2_scale, y, workspace, workspace_bytes, stream,
                combine_mode(num_tokens, hidden), "moe_fused_experts_from_logits"};
  MOE_TRY(check_experts(a));
  MOE_CHECK_ARG(logits_dtype == MOE_F32 || logits_dtype == MOE_BF16 || logits_dtype == MOE_F16,
                "moe_fused_experts_from_logits: logits dtype must be fp32, bf16 or fp16");
  MOE_CHECK_ARG(scoring == MOE_SCORE_SOFTMAX || scoring == MOE_SCORE_SIGMOID,
                "moe_fused_experts_from_logits: bad scoring %d", scoring);
  MOE_CHECK_ARG(top_k <= 32 && top_k <= num_experts, "moe_fused_experts_from_logits: top_k %d outside [1, min(E, 32)]",
                top_k);
  if (num_tokens == 0) return MOE_OK;
  MOE_CHECK_ARG(router_logits && topk_ids && topk_weights, "moe_fused_experts_from_logits: NULL pointer");
  if (one_launch(a) && decode_route_fits(num_experts, top_k, logits_dtype)) {
    // routing is phase 0 of the one-launch kernel
    cudaStream_t st = as_stream(stream);
    const DecodeRouting route{router_logits, logits_dtype, scoring == MOE_SCORE_SIGMOID, renormalize != 0,
                              topk_ids, topk_weights};
    MOE_CHECK_ARG(a.x && a.w13 && a.w2, "moe_fused_experts_from_logits: NULL input");
    MOE_TRY(record_stage(MOE_STAGE_ENTRY, st));
    MOE_TRY(decode_fused(x, x_dtype, num_tokens, hidden, w13, w2, num_experts, inter, nullptr, nullptr, top_k, y,
                         workspace, workspace_bytes, st, &route));
    for (int s = MOE_STAGE_ROUTED; s <= MOE_STAGE_DONE; ++s) MOE_TRY(record_stage(s, st));
    return MOE_OK;
  }
  MOE_TRY(moe_route_topk(router_logits, logits_dtype, num_tokens, num_experts, top_k, scoring, renormalize, topk_ids,
                         topk_weights, stream));
  return run_experts(a);
}

extern "C" size_t moe_fused_expert_rows_workspace_size(int64_t rows, int64_t hidden, int64_t inter, int num_experts,
                                                       int x_dtype, int w_dtype) {
  if (rows < 0 || hidden <= 0 || inter <= 0 || num_experts <= 0) return 0;
  if (dtype_size(x_dtype) == 0 || dtype_size(w_dtype) == 0) return 0;
  return fused_experts_ws(rows, hidden, inter, num_experts, 1, x_dtype, w_dtype, ExpertsOut::kScatterRows).bytes;
}

extern "C" int moe_fused_expert_rows(const void* x, int x_dtype, int64_t rows, int64_t hidden, const void* w13,
                                     const void* w2, int w_dtype, int num_experts, int64_t inter,
                                     const int32_t* expert_ids, const float* w13_scale, const float* w2_scale,
                                     void* out, void* workspace, size_t workspace_bytes, void* stream) {
  ExpertsArgs a{x, x_dtype, rows, hidden, w13, w2, w_dtype, num_experts, inter, nullptr, expert_ids,
                1, w13_scale, w2_scale, out, workspace, workspace_bytes, stream,
                ExpertsOut::kScatterRows, "moe_fused_expert_rows"};
  MOE_TRY(check_experts(a));
  return run_experts(a);
}
