// Tile schedule and routing align kernels.
//
//  * tile_schedule_kernel restates build_tile_schedule
//    (fused_moe_mlp_triton.py:91-119) on the device: one CTA scans the group
//    sizes and every thread resolves tiles with a binary search, so the
//    reference's eight small torch launches become one.
//  * align_* kernels implement the stable, block-padded counting sort of the
//    top-k slots by expert that the reference's callers get from an external
//    routing op (fused moe mlp triton.py:11-13): per-chunk warp histograms
//    (__match_any_sync), a per-expert scan over chunks, a per-expert scan
//    with padding to BLOCK_M, and a stable scatter.
#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "route.cuh"
#include "scan.cuh"

namespace moe {
namespace {

constexpr int kScanThreads = 1024;
constexpr int kChunk = 256;  // slots per align chunk (one warp, 8 rounds)

// ---------------------------------------------------------------------------
// build_tile_schedule (fused_moe_mlp_triton.py:91-119), bit-exact.
__global__ void __launch_bounds__(kScanThreads) tile_schedule_kernel(
    const void* __restrict__ gs_ptr, int gs_is64, int E, int BM, int64_t grid, int64_t* __restrict__ tile_expert,
    int64_t* __restrict__ tile_row_start, int64_t* __restrict__ tile_row_count, int32_t* __restrict__ table) {
  pdl_begin();
  extern __shared__ int64_t sh[];
  int64_t* offsets = sh;          // [E+1]  offsets[e] = sum gs[<e]
  int64_t* tcum = sh + (E + 1);   // [E+1]  tiles_cumsum
  __shared__ int64_t warp_sums[32];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int64_t g = gs_is64 ? reinterpret_cast<const int64_t*>(gs_ptr)[e]
                        : (int64_t) reinterpret_cast<const int32_t*>(gs_ptr)[e];
    if (g < 0) g = 0;  // negative counts are treated as empty groups
    offsets[e + 1] = g;
    tcum[e + 1] = (g + BM - 1) / BM;
  }
  if (threadIdx.x == 0) {
    offsets[0] = 0;
    tcum[0] = 0;
  }
  __syncthreads();
  smem_inclusive_scan<int64_t>(offsets + 1, E, warp_sums);
  smem_inclusive_scan<int64_t>(tcum + 1, E, warp_sums);

  const int64_t total_tiles = tcum[E];
  for (int64_t i = threadIdx.x; i < grid; i += blockDim.x) {
    // searchsorted(tcum[1:], i, right=True): number of e with tcum[e+1] <= i.
    int lo = 0, hi = E;  // answer in [0, E]
    while (lo < hi) {
      int mid = (lo + hi) >> 1;
      if (tcum[mid + 1] <= i) lo = mid + 1;
      else hi = mid;
    }
    const bool valid = lo < E;
    const int e = valid ? lo : E - 1;
    const int64_t local = i - tcum[e];
    const int64_t start = valid ? offsets[e] + local * BM : 0;
    int64_t count = offsets[e + 1] - start;
    count = count < 0 ? 0 : (count > BM ? BM : count);
    if (!valid) count = 0;
    if (tile_expert) tile_expert[i] = e;
    if (tile_row_start) tile_row_start[i] = start;
    if (tile_row_count) tile_row_count[i] = count;
    if (table && valid) {
      table[TileTable::start_off(E) + i] = (int32_t)start;
      table[TileTable::count_off(E, grid) + i] = (int32_t)count;
    }
  }
  if (table) {
    for (int e = threadIdx.x; e <= E; e += blockDim.x) table[TileTable::cum_off() + e] = (int32_t)tcum[e];
    if (threadIdx.x == 0) {
      table[0] = (int32_t)total_tiles;
      table[1] = (int32_t)offsets[E];
      table[2] = 0;
      table[3] = 0;
    }
  }
}

// ---------------------------------------------------------------------------
// Align, pass 1: per-chunk histogram (key E collects ids outside [0, E)).
__global__ void align_count_kernel(const int32_t* __restrict__ ids, int64_t S, int E,
                                   int32_t* __restrict__ chunk_hist) {
  pdl_begin();
  extern __shared__ int32_t hist[];  // [E+1]
  const int lane = threadIdx.x;
  for (int e = lane; e <= E; e += 32) hist[e] = 0;
  __syncwarp();
  const int64_t base = (int64_t)blockIdx.x * kChunk;
#pragma unroll 1
  for (int r = 0; r < kChunk / 32; ++r) {
    const int64_t s = base + r * 32 + lane;
    int key = -1;
    if (s < S) {
      const int id = ids[s];
      key = (id >= 0 && id < E) ? id : E;
    }
    const unsigned m = __match_any_sync(0xffffffffu, key);
    if (key >= 0 && lane == __ffs(m) - 1) hist[key] += __popc(m);
    __syncwarp();
  }
  int32_t* out = chunk_hist + (int64_t)blockIdx.x * (E + 1);
  for (int e = lane; e <= E; e += 32) out[e] = hist[e];
}

// Align, pass 2: exclusive scan of each expert column over chunks.
__global__ void __launch_bounds__(kScanThreads) align_colscan_kernel(const int32_t* __restrict__ chunk_hist,
                                                                     int num_chunks, int E,
                                                                     int32_t* __restrict__ chunk_base,
                                                                     int32_t* __restrict__ totals) {
  pdl_begin();
  __shared__ int32_t warp_sums[32];
  const int e = blockIdx.x;  // 0..E (E = dropped column)
  int32_t carry = 0;
  for (int c0 = 0; c0 < num_chunks; c0 += blockDim.x) {
    const int c = c0 + threadIdx.x;
    const int32_t v = (c < num_chunks) ? chunk_hist[(int64_t)c * (E + 1) + e] : 0;
    const int32_t incl = block_inclusive_scan<int32_t>(v, warp_sums);
    if (c < num_chunks) chunk_base[(int64_t)c * (E + 1) + e] = carry + incl - v;
    __shared__ int32_t last;
    if (threadIdx.x == blockDim.x - 1) last = incl;
    __syncthreads();
    carry += last;
    __syncthreads();
  }
  if (threadIdx.x == 0) totals[e] = carry;
}

// Align, pass 3: padded expert offsets, group sizes, tile table, pad fill.
__global__ void __launch_bounds__(kScanThreads) align_finalize_kernel(
    const int32_t* __restrict__ totals, int E, int BM, int64_t max_tiles, int32_t* __restrict__ group_sizes,
    int32_t* __restrict__ padded_offsets, int32_t* __restrict__ table, int32_t* __restrict__ sorted_slots) {
  pdl_begin();
  extern __shared__ int32_t sm[];
  int32_t* poff = sm;            // [E+1] padded offsets (exclusive)
  int32_t* tcum = sm + (E + 1);  // [E+1] tile cumsum (exclusive)
  __shared__ int32_t warp_sums[32];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int32_t c = totals[e];
    const int32_t t = (c + BM - 1) / BM;
    poff[e + 1] = t * BM;
    tcum[e + 1] = t;
    group_sizes[e] = c;
  }
  if (threadIdx.x == 0) {
    poff[0] = 0;
    tcum[0] = 0;
  }
  __syncthreads();
  smem_inclusive_scan<int32_t>(poff + 1, E, warp_sums);
  smem_inclusive_scan<int32_t>(tcum + 1, E, warp_sums);
  const int32_t ntiles = tcum[E];
  for (int e = threadIdx.x; e <= E; e += blockDim.x) {
    padded_offsets[e] = poff[e];
    table[TileTable::cum_off() + e] = tcum[e];
  }
  if (threadIdx.x == 0) {
    table[0] = ntiles;
    table[1] = poff[E];
    table[2] = totals[E];
    table[3] = 0;
  }
  for (int i = threadIdx.x; i < ntiles && i < max_tiles; i += blockDim.x) {
    int lo = 0, hi = E - 1;  // expert e with tcum[e] <= i < tcum[e+1]
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if (tcum[mid] <= i) lo = mid;
      else hi = mid - 1;
    }
    const int e = lo;
    const int j = i - tcum[e];
    const int32_t start = poff[e] + j * BM;
    const int32_t cnt = min(BM, totals[e] - j * BM);
    table[TileTable::start_off(E) + i] = start;
    table[TileTable::count_off(E, max_tiles) + i] = cnt;
    for (int r = cnt; r < BM; ++r) sorted_slots[start + r] = -1;
  }
}

// Align, pass 4: stable scatter of slots into their padded rows.
__global__ void align_scatter_kernel(const int32_t* __restrict__ ids, int64_t S, int E,
                                     const int32_t* __restrict__ chunk_base,
                                     const int32_t* __restrict__ padded_offsets,
                                     int32_t* __restrict__ sorted_slots, int32_t* __restrict__ slot_pos) {
  pdl_begin();
  extern __shared__ int32_t run[];  // [E]
  const int lane = threadIdx.x;
  const int32_t* cb = chunk_base + (int64_t)blockIdx.x * (E + 1);
  for (int e = lane; e < E; e += 32) run[e] = padded_offsets[e] + cb[e];
  __syncwarp();
  const int64_t base = (int64_t)blockIdx.x * kChunk;
  const unsigned lt_mask = (1u << lane) - 1u;
#pragma unroll 1
  for (int r = 0; r < kChunk / 32; ++r) {
    const int64_t s = base + r * 32 + lane;
    int key = -1;
    if (s < S) {
      const int id = ids[s];
      key = (id >= 0 && id < E) ? id : E;
    }
    const unsigned m = __match_any_sync(0xffffffffu, key);
    if (key >= 0 && key < E) {
      const int32_t pos = run[key] + __popc(m & lt_mask);
      sorted_slots[pos] = (int32_t)s;
      slot_pos[s] = pos;
    } else if (key == E) {
      slot_pos[s] = -1;
    }
    __syncwarp();
    if (key >= 0 && key < E && lane == __ffs(m) - 1) run[key] += __popc(m);
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Align in one CTA for small batches (S <= kAlignSmallSlots): the 32 warps
// play the chunks of the multi-kernel version — per-warp histograms, a scan
// of each expert column over the warps, the padded expert scan and tile
// table, then the stable scatter — all in shared memory, one launch.
constexpr int kAlignSmallSlots = 16384;

__global__ void __launch_bounds__(kScanThreads) align_small_kernel(
    const int32_t* __restrict__ ids, int64_t S, int E, int BM, int64_t max_tiles, int32_t* __restrict__ sorted_slots,
    int32_t* __restrict__ slot_pos, int32_t* __restrict__ group_sizes, int32_t* __restrict__ padded_offsets,
    int32_t* __restrict__ table) {
  pdl_begin();
  extern __shared__ int32_t sm[];
  constexpr int W = kScanThreads / 32;
  const int E1 = E + 1;
  int32_t* hist = sm;                // [W][E+1]: counts, then per-warp bases, then running positions
  int32_t* tot = sm + W * E1;        // [E+1] slots per expert (E: dropped)
  int32_t* poff = tot + E1;          // [E+1] padded offsets (exclusive)
  int32_t* tcum = poff + E1;         // [E+1] tile prefix (exclusive)
  __shared__ int32_t warp_sums[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < W * E1; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int64_t per = ((S + W - 1) / W + 31) / 32 * 32;  // slots per warp, whole rounds
  const int64_t lo = min(S, (int64_t)warp * per), hi = min(S, lo + per);
  int32_t* h = hist + warp * E1;
  for (int64_t b = lo; b < hi; b += 32) {
    const int64_t sl = b + lane;
    int key = -1;
    if (sl < hi) {
      const int id = ids[sl];
      key = (id >= 0 && id < E) ? id : E;
    }
    const unsigned m = __match_any_sync(0xffffffffu, key);
    if (key >= 0 && lane == __ffs(m) - 1) h[key] += __popc(m);
    __syncwarp();
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E1; e += blockDim.x) {  // exclusive scan of each column over the warps
    int run = 0;
    for (int w = 0; w < W; ++w) {
      const int v = hist[w * E1 + e];
      hist[w * E1 + e] = run;
      run += v;
    }
    tot[e] = run;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int t = (tot[e] + BM - 1) / BM;
    poff[e + 1] = t * BM;
    tcum[e + 1] = t;
    group_sizes[e] = tot[e];
  }
  if (threadIdx.x == 0) {
    poff[0] = 0;
    tcum[0] = 0;
  }
  __syncthreads();
  smem_inclusive_scan<int32_t>(poff + 1, E, warp_sums);
  smem_inclusive_scan<int32_t>(tcum + 1, E, warp_sums);
  const int32_t ntiles = tcum[E];
  for (int e = threadIdx.x; e <= E; e += blockDim.x) {
    padded_offsets[e] = poff[e];
    table[TileTable::cum_off() + e] = tcum[e];
  }
  if (threadIdx.x == 0) {
    table[0] = ntiles;
    table[1] = poff[E];
    table[2] = tot[E];
    table[3] = 0;
  }
  for (int i = threadIdx.x; i < ntiles && i < max_tiles; i += blockDim.x) {
    int a = 0, z = E - 1;
    while (a < z) {
      const int mid = (a + z + 1) >> 1;
      if (tcum[mid] <= i) a = mid;
      else z = mid - 1;
    }
    const int j = i - tcum[a];
    const int32_t start = poff[a] + j * BM;
    const int32_t cnt = min(BM, tot[a] - j * BM);
    table[TileTable::start_off(E) + i] = start;
    table[TileTable::count_off(E, max_tiles) + i] = cnt;
    for (int r = cnt; r < BM; ++r) sorted_slots[start + r] = -1;
  }
  for (int e = lane; e < E; e += 32) h[e] += poff[e];  // this warp's first padded row per expert
  __syncwarp();
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int64_t b = lo; b < hi; b += 32) {
    const int64_t sl = b + lane;
    int key = -1;
    if (sl < hi) {
      const int id = ids[sl];
      key = (id >= 0 && id < E) ? id : E;
    }
    const unsigned m = __match_any_sync(0xffffffffu, key);
    if (key >= 0 && key < E) {
      const int32_t pos = h[key] + __popc(m & lt_mask);
      sorted_slots[pos] = (int32_t)sl;
      slot_pos[sl] = pos;
    } else if (key == E) {
      slot_pos[sl] = -1;
    }
    __syncwarp();
    if (key >= 0 && key < E && lane == __ffs(m) - 1) h[key] += __popc(m);
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Router: logits [T, E] -> top-k ids and weights, one warp per token
// (route.cuh: ties to the lower expert id). When the tokens outnumber the
// warps that fit on the GPU at once, each warp takes R consecutive tokens
// at a time: their rows are loaded together and their selections interleave.
constexpr int kRouteMaxPerLane = 32;  // E <= 1024

template <typename T, int PER, int R>
__global__ void __launch_bounds__(256) route_topk_kernel(const T* __restrict__ logits, int64_t num_tokens, int E,
                                                         int k, int sigmoid, int renormalize,
                                                         int32_t* __restrict__ ids, float* __restrict__ wts) {
  pdl_begin();
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t t0 = warp * R; t0 < num_tokens; t0 += nwarps * R) {
    float v[R][PER];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t t = min(t0 + r, num_tokens - 1);  // a row past the end repeats the last one, not stored
      route_load<T, PER>(logits + t * E, E, lane, v[r]);
    }
    int id[R];
    float w[R];
    route_select<R, PER>(v, E, k, sigmoid, renormalize, lane, id, w);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t t = t0 + r;
      if (t < num_tokens && lane < k) {
        ids[t * k + lane] = id[r];
        wts[t * k + lane] = w[r];
      }
    }
  }
}

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" int moe_route_topk(const void* logits, int dtype, int64_t num_tokens, int num_experts, int top_k,
                              int scoring, int renormalize, int32_t* topk_ids, float* topk_weights, void* stream) {
  MOE_CHECK_ARG(num_tokens >= 0 && num_experts > 0 && num_experts <= 32 * kRouteMaxPerLane,
                "moe_route_topk: num_experts %d outside [1, %d]", num_experts, 32 * kRouteMaxPerLane);
  MOE_CHECK_ARG(top_k > 0 && top_k <= 32 && top_k <= num_experts, "moe_route_topk: top_k %d outside [1, min(E, 32)]",
                top_k);
  MOE_CHECK_ARG(scoring == MOE_SCORE_SOFTMAX || scoring == MOE_SCORE_SIGMOID, "moe_route_topk: bad scoring %d",
                scoring);
  if (num_tokens == 0) return MOE_OK;
  MOE_CHECK_ARG(logits && topk_ids && topk_weights, "moe_route_topk: NULL pointer");
  // one token per warp while every warp fits on the GPU at once (eight
  // 256-thread blocks per SM); above that four tokens per warp at a time
  // (E <= 256: their logits stay in registers)
  const int64_t resident_warps = (int64_t)num_sms() * 64;
  const int R = (num_tokens > resident_warps && num_experts <= 256) ? 4 : 1;
  int64_t blocks = ceil_div(ceil_div(num_tokens, (int64_t)R), (int64_t)8);
  const int64_t cap = (int64_t)num_sms() * 8;
  if (blocks > cap) blocks = cap;
  cudaStream_t st = as_stream(stream);
  const int sig = scoring == MOE_SCORE_SIGMOID;
#define ROUTE(TT, PER, RR)                                                                              \
  MOE_CUDA_TRY(launch_kernel(route_topk_kernel<TT, PER, RR>, dim3((unsigned)blocks), dim3(256), 0, st, \
                             static_cast<const TT*>(logits), num_tokens, num_experts, top_k, sig,       \
                             renormalize != 0, topk_ids, topk_weights))
#define ROUTE_T(TT)                                  \
  if (num_experts <= 32) {                           \
    if (R == 4) ROUTE(TT, 1, 4);                     \
    else ROUTE(TT, 1, 1);                            \
  } else if (num_experts <= 64) {                    \
    if (R == 4) ROUTE(TT, 2, 4);                     \
    else ROUTE(TT, 2, 1);                            \
  } else if (num_experts <= 128) {                   \
    if (R == 4) ROUTE(TT, 4, 4);                     \
    else ROUTE(TT, 4, 1);                            \
  } else if (num_experts <= 256) {                   \
    if (R == 4) ROUTE(TT, 8, 4);                     \
    else ROUTE(TT, 8, 1);                            \
  } else {                                           \
    ROUTE(TT, kRouteMaxPerLane, 1);                  \
  }
  if (dtype == MOE_F32) {
    ROUTE_T(float)
  } else if (dtype == MOE_BF16) {
    ROUTE_T(__nv_bfloat16)
  } else if (dtype == MOE_F16) {
    ROUTE_T(__half)
  } else {
    return set_error(MOE_ERR_UNSUPPORTED, "moe_route_topk: dtype %d not supported", dtype);
  }
#undef ROUTE_T
#undef ROUTE
  MOE_LAUNCH_CHECK("route_topk_kernel");
  return MOE_OK;
}

extern "C" int64_t moe_tile_grid(int64_t num_tokens, int num_experts, int block_m) {
  if (block_m <= 0 || num_tokens < 0 || num_experts <= 0) return -1;
  return ceil_div(num_tokens, block_m) + num_experts;
}

extern "C" int64_t moe_tile_table_ints(int num_experts, int64_t max_tiles) {
  return TileTable::ints(num_experts, max_tiles);
}

extern "C" int moe_tile_schedule(const void* group_sizes, int gs_dtype, int num_experts, int64_t num_tokens,
                                 int block_m, int64_t* tile_expert, int64_t* tile_row_start,
                                 int64_t* tile_row_count, int32_t* tile_table, void* stream) {
  MOE_CHECK_ARG(group_sizes != nullptr, "moe_tile_schedule: group_sizes is NULL");
  MOE_CHECK_ARG(gs_dtype == MOE_I32 || gs_dtype == MOE_I64, "moe_tile_schedule: group_sizes must be int32/int64");
  MOE_CHECK_ARG(num_experts > 0 && num_experts <= 4096, "moe_tile_schedule: num_experts %d outside [1, 4096]",
                num_experts);
  MOE_CHECK_ARG(block_m > 0, "moe_tile_schedule: block_m must be positive");
  MOE_CHECK_ARG(num_tokens >= 0 && num_tokens < (int64_t(1) << 31), "moe_tile_schedule: num_tokens out of range");
  const int64_t grid = moe_tile_grid(num_tokens, num_experts, block_m);
  const size_t smem = 2 * (num_experts + 1) * sizeof(int64_t);
  if (smem > 48 * 1024)
    MOE_CUDA_TRY(cudaFuncSetAttribute(tile_schedule_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  MOE_CUDA_TRY(launch_kernel(tile_schedule_kernel, dim3(1), dim3(kScanThreads), smem, as_stream(stream),
                             group_sizes, gs_dtype == MOE_I64, num_experts, block_m, grid, tile_expert,
                             tile_row_start, tile_row_count, tile_table));
  MOE_LAUNCH_CHECK("tile_schedule_kernel");
  return MOE_OK;
}

namespace {
struct AlignWs {
  int64_t chunks;
  size_t hist_off, base_off, totals_off, bytes;
};
AlignWs align_ws(int64_t S, int E) {
  AlignWs w;
  w.chunks = ceil_div(S, kChunk);
  const size_t col = (size_t)(E + 1) * sizeof(int32_t);
  w.hist_off = 0;
  w.base_off = align_up(w.chunks * col, 256);
  w.totals_off = w.base_off + align_up(w.chunks * col, 256);
  w.bytes = w.totals_off + align_up(col, 256);
  return w;
}
}  // namespace

extern "C" int64_t moe_align_capacity(int64_t num_slots, int num_experts, int block_m) {
  if (num_slots < 0 || num_experts <= 0 || block_m <= 0) return -1;
  // every non-empty expert's segment is padded by at most block_m - 1 rows,
  // and at most min(E, slots) experts are non-empty; round the total up to
  // whole tiles so TMA boxes of block_m rows stay in bounds.
  const int64_t nonempty = std::min<int64_t>(num_experts, num_slots);
  int64_t cap = num_slots + nonempty * (block_m - 1);
  return ceil_div(cap, block_m) * block_m;
}

extern "C" size_t moe_align_workspace_size(int64_t num_tokens, int top_k, int num_experts, int block_m) {
  (void)block_m;
  if (num_tokens < 0 || top_k <= 0 || num_experts <= 0) return 0;
  return align_ws(num_tokens * top_k, num_experts).bytes;
}

namespace {
// One-CTA align for S <= kAlignSmallSlots slots over at most 1024 experts:
// everything in shared memory, no scratch.
bool align_is_small(int64_t S, int E) { return S <= kAlignSmallSlots && E <= 1024; }

int launch_align_small(const int32_t* topk_ids, int64_t S, int E, int block_m, int32_t* sorted_slots,
                       int32_t* slot_pos, int32_t* group_sizes, int32_t* padded_offsets, int32_t* tile_table,
                       cudaStream_t st) {
  const int64_t max_tiles = moe_align_capacity(S, E, block_m) / block_m;
  const size_t smem = ((size_t)(kScanThreads / 32) + 3) * (E + 1) * sizeof(int32_t);
  if (smem > 48 * 1024)
    MOE_CUDA_TRY(cudaFuncSetAttribute(align_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  MOE_CUDA_TRY(launch_kernel(align_small_kernel, dim3(1), dim3(kScanThreads), smem, st, topk_ids, S, E, block_m,
                             max_tiles, sorted_slots, slot_pos, group_sizes, padded_offsets, tile_table));
  MOE_LAUNCH_CHECK("align_small_kernel");
  return MOE_OK;
}

// The four-kernel align (chunk histograms, column scan, expert scan with
// padding and tile table, stable scatter) with its scratch at `scratch`
// (align_ws(S, E).bytes, laid out by align_ws).
int launch_align_chunked(const int32_t* topk_ids, int64_t S, int E, int block_m, int32_t* sorted_slots,
                         int32_t* slot_pos, int32_t* group_sizes, int32_t* padded_offsets, int32_t* tile_table,
                         void* scratch, cudaStream_t st) {
  const AlignWs w = align_ws(S, E);
  char* ws = static_cast<char*>(scratch);
  int32_t* hist = reinterpret_cast<int32_t*>(ws + w.hist_off);
  int32_t* base = reinterpret_cast<int32_t*>(ws + w.base_off);
  int32_t* totals = reinterpret_cast<int32_t*>(ws + w.totals_off);
  const int64_t max_tiles = moe_align_capacity(S, E, block_m) / block_m;
  const size_t hsmem = (E + 1) * sizeof(int32_t);
  if (w.chunks > 0) {
    MOE_CUDA_TRY(launch_kernel(align_count_kernel, dim3((unsigned)w.chunks), dim3(32), hsmem, st, topk_ids, S, E,
                               hist));
    MOE_LAUNCH_CHECK("align_count_kernel");
  }
  MOE_CUDA_TRY(launch_kernel(align_colscan_kernel, dim3(E + 1), dim3(kScanThreads), 0, st, hist, (int)w.chunks, E,
                             base, totals));
  MOE_LAUNCH_CHECK("align_colscan_kernel");
  MOE_CUDA_TRY(launch_kernel(align_finalize_kernel, dim3(1), dim3(kScanThreads), 2 * hsmem, st, totals, E, block_m,
                             max_tiles, group_sizes, padded_offsets, tile_table, sorted_slots));
  MOE_LAUNCH_CHECK("align_finalize_kernel");
  if (w.chunks > 0) {
    MOE_CUDA_TRY(launch_kernel(align_scatter_kernel, dim3((unsigned)w.chunks), dim3(32), hsmem, st, topk_ids, S, E,
                               base, padded_offsets, sorted_slots, slot_pos));
    MOE_LAUNCH_CHECK("align_scatter_kernel");
  }
  return MOE_OK;
}
}  // namespace

extern "C" int moe_align(const int32_t* topk_ids, int64_t num_tokens, int top_k, int num_experts, int block_m,
                         int32_t* sorted_slots, int32_t* slot_pos, int32_t* group_sizes, int32_t* padded_offsets,
                         int32_t* tile_table, void* workspace, size_t workspace_bytes, void* stream) {
  MOE_CHECK_ARG(num_tokens >= 0 && top_k > 0, "moe_align: bad num_tokens/top_k");
  MOE_CHECK_ARG(num_experts > 0 && num_experts <= 4096, "moe_align: num_experts %d outside [1, 4096]",
                num_experts);
  MOE_CHECK_ARG(block_m > 0 && block_m <= 1024, "moe_align: block_m %d outside [1, 1024]", block_m);
  const int64_t S = num_tokens * top_k;
  MOE_CHECK_ARG(S < (int64_t(1) << 30), "moe_align: too many slots");
  MOE_CHECK_ARG(S == 0 || (topk_ids && slot_pos), "moe_align: NULL ids/slot_pos");
  MOE_CHECK_ARG(sorted_slots && group_sizes && padded_offsets && tile_table, "moe_align: NULL output");
  const AlignWs w = align_ws(S, num_experts);
  if (workspace_bytes < w.bytes || (w.bytes && !workspace))
    return set_error(MOE_ERR_WORKSPACE, "moe_align: workspace %zu < %zu bytes", workspace_bytes, w.bytes);
  if (align_is_small(S, num_experts))
    return launch_align_small(topk_ids, S, num_experts, block_m, sorted_slots, slot_pos, group_sizes,
                              padded_offsets, tile_table, as_stream(stream));
  return launch_align_chunked(topk_ids, S, num_experts, block_m, sorted_slots, slot_pos, group_sizes, padded_offsets,
                              tile_table, workspace, as_stream(stream));
}

// ---------------------------------------------------------------------------
// moe_align_static: moe_align without a workspace argument. Batches the
// one-CTA kernel handles (at most 16384 slots over at most 1024 experts) need
// no scratch at all; larger ones run the four align kernels with their
// scratch in a file-scope device array instead of a caller workspace, for
// callers that cannot allocate device memory. Nothing in the scratch has to
// start at zero: every histogram, base and total the kernels read is written
// earlier in the same call. Calls that overlap on the GPU share (and race on)
// the array.
namespace {
static __device__ __align__(256) unsigned char g_align_scratch[MOE_ALIGN_STATIC_SCRATCH_BYTES];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// The calling thread's current CUDA context (driver API, reached through the
// runtime's entry-point query so the library links no libcuda).
int current_context(CUcontext* ctx) {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (CtxGetCurrentFn) nullptr;
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  if (!fn) return set_error(MOE_ERR_CUDA, "moe_align_static: cuCtxGetCurrent unavailable");
  if (fn(ctx) != CUDA_SUCCESS) return set_error(MOE_ERR_CUDA, "moe_align_static: cuCtxGetCurrent failed");
  return MOE_OK;
}

struct ScratchAddr {
  CUcontext ctx = nullptr;
  void* ptr = nullptr;
};
std::mutex g_align_scratch_mu;
ScratchAddr g_align_scratch_addr[64];

// Device address of g_align_scratch on the current device. In host code the
// symbol is only a host-side stand-in, so the address is looked up with the
// device current, once per device and context, and cached; a new context on
// the device (after cudaDeviceReset, say) loads the module afresh, possibly
// elsewhere, so the lookup is redone then.
int align_scratch_address(void** out) {
  int dev = 0;
  MOE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(MOE_ERR_UNSUPPORTED, "moe_align_static: device %d >= 64", dev);
  CUcontext ctx = nullptr;
  MOE_TRY(current_context(&ctx));
  std::lock_guard<std::mutex> lock(g_align_scratch_mu);
  ScratchAddr& a = g_align_scratch_addr[dev];
  if (!ctx || !a.ptr || a.ctx != ctx) {
    // no context current on this thread yet, or a different one: the lookup
    // makes the device's primary context current and loads the module
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_align_scratch);
    if (e != cudaSuccess || !p)
      return set_error(MOE_ERR_CUDA, "moe_align_static: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    MOE_TRY(current_context(&ctx));
    a.ctx = ctx;
    a.ptr = p;
  }
  *out = a.ptr;
  return MOE_OK;
}
}  // namespace

extern "C" int moe_align_static(const int32_t* topk_ids, int64_t num_tokens, int top_k, int num_experts,
                                int block_m, int32_t* sorted_slots, int32_t* slot_pos, int32_t* group_sizes,
                                int32_t* padded_offsets, int32_t* tile_table, void* stream) {
  MOE_CHECK_ARG(num_tokens >= 0 && top_k > 0, "moe_align_static: bad num_tokens/top_k");
  MOE_CHECK_ARG(num_experts > 0 && num_experts <= 4096, "moe_align_static: num_experts %d outside [1, 4096]",
                num_experts);
  MOE_CHECK_ARG(block_m > 0 && block_m <= 1024, "moe_align_static: block_m %d outside [1, 1024]", block_m);
  const int64_t S = num_tokens * top_k;
  MOE_CHECK_ARG(S < (int64_t(1) << 30), "moe_align_static: too many slots");
  MOE_CHECK_ARG(S == 0 || (topk_ids && slot_pos), "moe_align_static: NULL ids/slot_pos");
  MOE_CHECK_ARG(sorted_slots && group_sizes && padded_offsets && tile_table, "moe_align_static: NULL output");
  const AlignWs w = align_ws(S, num_experts);
  MOE_CHECK_ARG(w.bytes <= MOE_ALIGN_STATIC_SCRATCH_BYTES,
                "moe_align_static: %lld slots over %d experts need %zu bytes of scratch, more than the static "
                "%u-byte array; use moe_align with a workspace",
                (long long)S, num_experts, w.bytes, (unsigned)MOE_ALIGN_STATIC_SCRATCH_BYTES);
  if (align_is_small(S, num_experts))
    return launch_align_small(topk_ids, S, num_experts, block_m, sorted_slots, slot_pos, group_sizes,
                              padded_offsets, tile_table, as_stream(stream));
  void* scratch = nullptr;
  MOE_TRY(align_scratch_address(&scratch));
  return launch_align_chunked(topk_ids, S, num_experts, block_m, sorted_slots, slot_pos, group_sizes, padded_offsets,
                              tile_table, scratch, as_stream(stream));
}
