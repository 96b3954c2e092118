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

int record_stage(int stage, cudaStream_t st) {
  if (g_stage_events && stage < g_num_stage_events && g_stage_events[stage])
    MOE_CUDA_TRY(cudaEventRecord(static_cast<cudaEvent_t>(g_stage_events[stage]), st));
  return MOE_OK;
}
}  // namespace

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

struct FusedExpertsWs {
  int64_t S, cap, max_tiles;
  size_t align_bytes;
  size_t align, sorted, slot_pos, gs, poff, table, xp, xs, h, hq, hs, y32, bytes;
};
FusedExpertsWs fused_experts_ws(int64_t T, int64_t H, int64_t I, int E, int k, int x_dtype, int w_dtype) {
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
  w.y32 = c.take(x_dtype == MOE_F32 ? 0 : (size_t)T * H * sizeof(float));
  w.bytes = c.off;
  return w;
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
  MOE_CHECK_ARG(out != nullptr, "moe_fused_mlp: out is NULL");
  if (num_tokens == 0) return MOE_OK;
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
  MOE_CUDA_TRY(cudaMemsetAsync(out, 0, (size_t)num_tokens * hidden * dtype_size(dtype), st));
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
  return fused_experts_ws(num_tokens, hidden, inter, num_experts, top_k, x_dtype, w_dtype).bytes;
}

extern "C" int moe_fused_experts(const void* x, int x_dtype, int64_t num_tokens, int64_t hidden, const void* w13,
                                 const void* w2, int w_dtype, int num_experts, int64_t inter,
                                 const float* topk_weights, const int32_t* topk_ids, int top_k,
                                 const float* w13_scale, const float* w2_scale, void* y, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  MOE_CHECK_ARG(x_dtype == MOE_BF16 || x_dtype == MOE_F16 || x_dtype == MOE_F32,
                "moe_fused_experts: x dtype must be bf16, fp16 or fp32");
  MOE_CHECK_ARG(w_dtype == x_dtype || w_dtype == MOE_I8,
                "moe_fused_experts: weights must share x's dtype or be int8 (w8a8)");
  MOE_CHECK_ARG(!(w_dtype == MOE_I8 && x_dtype == MOE_F32), "moe_fused_experts: w8a8 takes bf16/fp16 activations");
  if (w_dtype == MOE_I8) MOE_CHECK_ARG(w13_scale && w2_scale, "moe_fused_experts: int8 weights need scales");
  MOE_CHECK_ARG(num_tokens >= 0 && hidden > 0 && inter > 0 && num_experts > 0 && top_k > 0,
                "moe_fused_experts: bad sizes");
  MOE_CHECK_ARG(y != nullptr, "moe_fused_experts: y is NULL");
  if (num_tokens == 0) return MOE_OK;
  MOE_CHECK_ARG(x && w13 && w2 && topk_weights && topk_ids, "moe_fused_experts: NULL input");
  const FusedExpertsWs w = fused_experts_ws(num_tokens, hidden, inter, num_experts, top_k, x_dtype, w_dtype);
  if (workspace_bytes < w.bytes || !workspace)
    return set_error(MOE_ERR_WORKSPACE, "moe_fused_experts: workspace %zu < %zu bytes", workspace_bytes, w.bytes);
  char* ws = static_cast<char*>(workspace);
  int32_t* sorted = reinterpret_cast<int32_t*>(ws + w.sorted);
  int32_t* slot_pos = reinterpret_cast<int32_t*>(ws + w.slot_pos);
  int32_t* gs = reinterpret_cast<int32_t*>(ws + w.gs);
  int32_t* poff = reinterpret_cast<int32_t*>(ws + w.poff);
  int32_t* table = reinterpret_cast<int32_t*>(ws + w.table);
  const bool q = (w_dtype == MOE_I8);
  const int h_dtype = (x_dtype == MOE_F32) ? MOE_F32 : (q ? MOE_BF16 : x_dtype);
  cudaStream_t st = as_stream(stream);

  MOE_TRY(record_stage(MOE_STAGE_ENTRY, st));
  MOE_TRY(moe_align(topk_ids, num_tokens, top_k, num_experts, kBlockM, sorted, slot_pos, gs, poff, table,
                    ws + w.align, w.align_bytes, stream));
  MOE_TRY(record_stage(MOE_STAGE_ROUTED, st));
  const int32_t* rows_dev = table + 1;  // padded rows in use
  void* xp = ws + w.xp;
  float* xs = q ? reinterpret_cast<float*>(ws + w.xs) : nullptr;
  MOE_TRY(moe_gather_rows(x, x_dtype, hidden, sorted, top_k, w.cap, rows_dev, xp, q ? MOE_I8 : x_dtype, xs, stream));
  MOE_TRY(record_stage(MOE_STAGE_GATHERED, st));
  void* h = ws + w.h;
  MOE_TRY(moe_gemm1_swiglu(xp, q ? MOE_I8 : x_dtype, w.cap, hidden, w13, num_experts, inter, xs, w13_scale, table,
                           w.max_tiles, h, h_dtype, stream));
  MOE_TRY(record_stage(MOE_STAGE_GEMM1, st));
  const void* a2 = h;
  float* hs = nullptr;
  if (q) {
    int8_t* hq = reinterpret_cast<int8_t*>(ws + w.hq);
    hs = reinterpret_cast<float*>(ws + w.hs);
    MOE_TRY(moe_quant_rows(h, h_dtype, w.cap, inter, rows_dev, hq, hs, stream));
    a2 = hq;
  }
  float* acc = (x_dtype == MOE_F32) ? static_cast<float*>(y) : reinterpret_cast<float*>(ws + w.y32);
  MOE_CUDA_TRY(cudaMemsetAsync(acc, 0, (size_t)num_tokens * hidden * sizeof(float), st));
  MOE_TRY(record_stage(MOE_STAGE_PRE_GEMM2, st));
  MOE_TRY(moe_gemm2(a2, q ? MOE_I8 : h_dtype, w.cap, inter, w2, num_experts, hidden, hs, w2_scale, table,
                    w.max_tiles, MOE_EPI_COMBINE_ADD, sorted, topk_weights, top_k, acc, MOE_F32, num_tokens, stream));
  MOE_TRY(record_stage(MOE_STAGE_GEMM2, st));
  if (x_dtype != MOE_F32) MOE_TRY(moe_convert_f32(acc, num_tokens * hidden, y, x_dtype, stream));
  MOE_TRY(record_stage(MOE_STAGE_DONE, st));
  return MOE_OK;
}
