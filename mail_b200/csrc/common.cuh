// Internal helpers shared by the MoE translation units: status/error
// reporting, dtype sizes, the compact tile table, and the device error flag.
#pragma once
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/moe_b200.h"

namespace moe {

constexpr int kBlockM = 128;  // rows per M tile (UMMA M)

// Records a message for moe_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);

#define MOE_CHECK_ARG(cond, ...)                                   \
  do {                                                             \
    if (!(cond)) return ::moe::set_error(MOE_ERR_INVALID_ARG, __VA_ARGS__); \
  } while (0)

#define MOE_CUDA_TRY(expr)                                                                       \
  do {                                                                                           \
    cudaError_t e_ = (expr);                                                                     \
    if (e_ != cudaSuccess)                                                                       \
      return ::moe::set_error(MOE_ERR_CUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_), \
                              __FILE__, __LINE__);                                               \
  } while (0)

// Counts one kernel launch (moe_launch_count).
void note_launch();

// Records the caller's profiling event for stage `stage` (moe_set_stage_events).
int record_stage(int stage, cudaStream_t st);

#define MOE_LAUNCH_CHECK(name)                                                                   \
  do {                                                                                           \
    cudaError_t e_ = cudaGetLastError();                                                         \
    if (e_ != cudaSuccess)                                                                       \
      return ::moe::set_error(MOE_ERR_CUDA, "launch of %s failed: %s", name, cudaGetErrorString(e_)); \
    ::moe::note_launch();                                                                        \
  } while (0)

#define MOE_TRY(expr)            \
  do {                           \
    int s_ = (expr);             \
    if (s_ != MOE_OK) return s_; \
  } while (0)

inline int dtype_size(int dt) {
  switch (dt) {
    case MOE_F32: return 4;
    case MOE_F16: return 2;
    case MOE_BF16: return 2;
    case MOE_I8: return 1;
    case MOE_I32: return 4;
    case MOE_I64: return 8;
    default: return 0;
  }
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Compact int32 tile table written by the schedule/align kernels and read by
// the GEMMs:
//   [0] number of valid M tiles        [1] rows covered (padded rows for align)
//   [2] dropped slots (align)          [3] reserved
//   [4 .. 4+E]          tile_cumsum[E+1] (tiles of expert e are [cum[e], cum[e+1]))
//   [5+E .. 5+E+T)      row_start[T]
//   [5+E+T .. 5+E+2T)   row_count[T]           (T = max_tiles)
struct TileTable {
  static constexpr int kHeader = 4;
  __host__ __device__ static int64_t ints(int E, int64_t max_tiles) { return kHeader + (E + 1) + 2 * max_tiles; }
  __host__ __device__ static int64_t cum_off() { return kHeader; }
  __host__ __device__ static int64_t start_off(int E) { return kHeader + E + 1; }
  __host__ __device__ static int64_t count_off(int E, int64_t max_tiles) { return kHeader + E + 1 + max_tiles; }
};

// Device error codes latched by the GEMM kernels (first error wins):
// 1 = TMA producer wait, 2 = MMA issuer wait, 3 = epilogue wait, 4 = drain wait.
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Internal GEMM2 epilogue (expert-parallel return path): row r's result goes
// to peer_out[meta >> 24] at row meta & 0xFFFFFF, meta = row_map[r] (< 0: skip).
constexpr int kEpiScatterPeer = 3;

// Operand roles and K splits of one MoE layer's two grouped GEMMs
// (moe_gemm.cu). swap: few token rows per expert, so the weights are the
// MMA's 128-row operand and the tokens its N operand (moe_gemm_swap.cuh).
struct GemmPlan {
  bool swap = false;         // gate_up GEMM swapped
  bool swap2 = false;        // down GEMM swapped as well
  int nmax = 128;            // token rows per swapped work item (32 or 128)
  int splits1 = 1;           // K splits of the gate_up GEMM (swapped)
  int splits2 = 1;           // K splits of the down GEMM (swapped, combine epilogue only)
  size_t partial_bytes = 0;  // gate_up split-K slots
  size_t counter_bytes = 0;  // gate_up split-K counts (zeroed before the launch)
};

// Plan for `slots` routed rows over `num_experts` experts (max_tiles M tiles of
// 128 rows); combine: the down GEMM uses the additive combine epilogue.
GemmPlan gemm_plan(int64_t slots, int num_experts, int64_t max_tiles, int64_t hidden, int64_t inter, int dtype,
                   bool combine);

// Output conversion fused into the swapped down GEMM's combine epilogue: when
// the last contribution to a (token, 32-output-feature group) of the fp32
// accumulator has been added (a count per group reaching the token's routed
// slots x K splits), the warp that added it converts the group to `out`.
struct FusedConvert {
  void* out;               // [T, H] in dtype
  int dtype;
  int32_t* counters;       // [T][H / 32 rounded up to 4 per 128], zero on entry
  const int32_t* kvalid;   // [T] routed slots per token
};

// moe_gemm1_swiglu / moe_gemm2 with an explicit plan (nullptr: the row-major
// kernels, or the swapped one when MOE_OPT_GEMM_SWAP_AB forces it) and, for a
// gate_up split, its workspace (partial slots and zeroed counters).
int gemm1_swiglu_planned(const void* a, int dtype, int64_t a_rows, int64_t hidden, const void* w13, int num_experts,
                         int64_t inter, const float* a_scale, const float* w13_scale, const int32_t* tile_table,
                         int64_t max_tiles, void* h, int h_dtype, const GemmPlan* plan, void* partial,
                         int32_t* counters, cudaStream_t stream);
int gemm2_planned(const void* h, int dtype, int64_t h_rows, int64_t inter, const void* w2, int num_experts,
                  int64_t hidden, const float* h_scale, const float* w2_scale, const int32_t* tile_table,
                  int64_t max_tiles, int epilogue, const int32_t* row_map, const float* row_weight, int top_k,
                  void* out, int out_dtype, int64_t out_rows, const GemmPlan* plan, cudaStream_t stream,
                  const FusedConvert* convert = nullptr);

// Down GEMM whose epilogue stores each output row into the buffer of the rank
// that sent the row (peer pointers, NVLink stores). Defined in moe_gemm.cu.
int gemm2_scatter_peer(const void* h, int dtype, int64_t h_rows, int64_t inter, const void* w2, int num_experts,
                       int64_t hidden, const float* h_scale, const float* w2_scale, const int32_t* tile_table,
                       int64_t max_tiles, const int32_t* row_meta, void* const* peer_out, int num_peers,
                       int64_t peer_rows, int out_dtype, cudaStream_t stream);

// Programmatic dependent launch (PDL). Every kernel of this library starts
// with pdl_begin(): it waits until the grids launched before it in the stream
// have completed and their memory is visible, then lets the next grid in the
// stream be scheduled, so that grid's launch and prologue overlap this one.
// A grid launched without the programmatic-serialisation attribute returns
// from the wait at once. Nothing before the wait touches global memory.
__device__ __forceinline__ void pdl_begin() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Kernel clocks (MOE_OPT_KERNEL_CLOCKS): per kernel class, the busy time of
// every launch measured on the device with the global nanosecond timer —
// from the moment the first CTA is past its wait on the preceding grids to
// the moment the last CTA finishes — summed over launches. The first CTA to
// arrive stamps the start; the last to finish (a completion count over the
// grid) adds end - start and re-arms the record for the next launch. Two
// atomics per CTA; launches of one class never overlap (stream order).
struct KernelClock {
  unsigned long long start;
  unsigned long long total_ns;
  unsigned long long launches;
  unsigned int started;
  unsigned int finished;
};

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Call after pdl_begin(), from every CTA.
__device__ __forceinline__ void clock_begin(KernelClock* c) {
  if (c != nullptr && threadIdx.x == 0 && atomicAdd(&c->started, 1u) == 0u) atomicExch(&c->start, global_ns());
}

// Call at the very end, after a __syncthreads(), from every CTA.
__device__ __forceinline__ void clock_end(KernelClock* c) {
  if (c == nullptr || threadIdx.x != 0) return;
  __threadfence();
  const unsigned int nblocks = gridDim.x * gridDim.y * gridDim.z;
  if (atomicAdd(&c->finished, 1u) == nblocks - 1u) {
    __threadfence();
    const unsigned long long t = global_ns();
    const unsigned long long s = atomicAdd(&c->start, 0ull);
    atomicAdd(&c->total_ns, t - s);
    atomicAdd(&c->launches, 1ull);
    atomicExch(&c->started, 0u);
    atomicExch(&c->finished, 0u);
    __threadfence();
  }
}

// Whether launches carry the programmatic-serialisation attribute
// (MOE_OPT_PDL, default on). Defined in moe_gemm.cu.
bool pdl_enabled();

// cudaLaunchKernelEx with the PDL attribute when enabled.
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                          Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  if (pdl_enabled()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Zeroes `bytes` of device memory on `st` (a kernel launch: moe_rows.cu).
int zero_fill(void* dst, size_t bytes, cudaStream_t st);

// moe_gather_rows, with padding rows zero-filled or left untouched (moe_rows.cu).
int gather_rows(const void* src, int src_dtype, int64_t cols, const int32_t* sorted_slots, int top_k, int64_t rows,
                const int32_t* rows_dev, void* dst, int dst_dtype, float* dst_scale, bool zero_pad, void* stream);

// Decode-sized layer prep in one launch (moe_prep.cu): the align, the
// permuting gather (+ int8 quantisation), and zero fills of two buffers.
constexpr int64_t kPrepMaxSlots = 4096;
bool prep_small_fits(int64_t slots, int num_experts);
int prep_small(const int32_t* topk_ids, int64_t num_tokens, int top_k, int num_experts, int block_m,
               const void* x, int x_dtype, int64_t hidden, void* xp, bool quant, float* xs, int32_t* sorted_slots,
               int32_t* slot_pos, int32_t* group_sizes, int32_t* padded_offsets, int32_t* tile_table,
               void* zero_a, size_t zero_a_bytes, void* zero_b, size_t zero_b_bytes, int32_t* kvalid, void* y,
               cudaStream_t st);


// The whole top-k layer for at most 16 tokens (and 128 routed slots) in one
// persistent launch (moe_decode.cuh): routing, gate_up, down + combine,
// conversion, separated by device-wide barriers (MOE_OPT_DECODE_FUSED).
bool decode_fused_fits(int64_t T, int k, int E, int64_t H, int64_t I, int x_dtype, int w_dtype);
size_t decode_fused_workspace(int64_t T, int k, int E, int64_t H, int64_t I, int dtype);
// Routing inside the one-launch kernel: the router logits [T, E] in, the
// top-k ids and weights [T, k] out (decode_fused's topk_weights / topk_ids
// are then not read).
struct DecodeRouting {
  const void* logits;
  int dtype;  // MOE_F32, MOE_BF16 or MOE_F16
  int sigmoid, renormalize;
  int32_t* ids_out;
  float* wts_out;
};
bool decode_route_fits(int E, int k, int logits_dtype);
int decode_fused(const void* x, int dtype, int64_t T, int64_t H, const void* w13, const void* w2, int E, int64_t I,
                 const float* topk_weights, const int32_t* topk_ids, int k, void* y, void* workspace,
                 size_t workspace_bytes, cudaStream_t st, const DecodeRouting* route = nullptr);

// Token-order scatter of the routed rows (+ per-token int8 quantisation):
// dst[slot_pos[t * k + j]] = row t of src, each row read once (moe_rows.cu).
bool scatter_rows_fits(int64_t cols);
int scatter_rows(const void* src, int src_dtype, int64_t cols, const int32_t* slot_pos, int top_k, int64_t T,
                 void* dst, int dst_dtype, float* dst_scale, cudaStream_t st);

// SM count of the current device (queried once per device; threads may race
// to fill the cache with the same value).
inline int num_sms() {
  static std::atomic<int> cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

}  // namespace moe
