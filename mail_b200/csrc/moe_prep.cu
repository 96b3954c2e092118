// Decode-sized layer prep in one launch.
//
// For a small batch (at most kPrepMaxSlots routed slots over at most 1024
// experts) the top-k op's work before the gate_up GEMM — the routing align,
// the permuting gather (with the per-token int8 quantisation for w8a8), and
// the clearing of the fp32 combine accumulator and of the GEMMs' split-K
// counters — is a few microseconds of work spread over four launches, each
// costing a launch and a dependency wait. Here it is one kernel:
//
//   * every CTA loads all the slot ids into shared memory and computes the
//     stable, block-padded align there (per-warp histograms of contiguous
//     slot ranges with __match_any_sync, a column scan over the warps, the
//     padded expert scan) — the same arithmetic as the align kernels, so the
//     outputs are bit-identical to moe_align's;
//   * CTA 0 writes the align outputs (group sizes, padded offsets, tile
//     table, slot positions, and the slot of every routed row; padding rows
//     of sorted_slots are not written, the GEMMs never read them);
//   * every CTA gathers its share of the routed rows (one warp per slot,
//     16-byte accesses; int8 rows get absmax / 127 scales) and clears its
//     share of the two zero-filled buffers;
//   * optionally (kvalid != NULL) the routed-slot count of every token, which
//     the down GEMM's fused output conversion waits for, with a zero output
//     row written here for a token whose slots were all dropped.
#include "common.cuh"
#include "rows.cuh"
#include "scan.cuh"

namespace moe {
namespace {
using namespace rows;

constexpr int kPrepThreads = 256;
constexpr int kPrepWarps = kPrepThreads / 32;

template <typename Tin, bool QUANT>
__global__ void __launch_bounds__(kPrepThreads) prep_small_kernel(
    const int32_t* __restrict__ ids, int64_t S, int k, int E, int BM, int64_t max_tiles, const Tin* __restrict__ x,
    int64_t H, void* __restrict__ xp, float* __restrict__ xs, int32_t* __restrict__ sorted,
    int32_t* __restrict__ slot_pos, int32_t* __restrict__ gs, int32_t* __restrict__ poff_out,
    int32_t* __restrict__ table, uint4* __restrict__ zero_a, int64_t zero_a16, uint4* __restrict__ zero_b,
    int64_t zero_b16, int32_t* __restrict__ kvalid, Tin* __restrict__ y) {
  pdl_begin();
  extern __shared__ int32_t sm[];
  const int E1 = E + 1;
  int32_t* s_ids = sm;                    // [S]
  int32_t* s_pos = s_ids + S;             // [S] padded row of each slot (-1: dropped)
  int32_t* hist = s_pos + S;              // [W][E+1]: counts, then per-warp bases, then running positions
  int32_t* tot = hist + kPrepWarps * E1;  // [E+1] slots per expert (E: dropped)
  int32_t* poff = tot + E1;               // [E+1] padded offsets (exclusive)
  int32_t* tcum = poff + E1;              // [E+1] tile prefix (exclusive)
  __shared__ int32_t warp_sums[32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  for (int64_t i = tid; i < S; i += blockDim.x) s_ids[i] = ids[i];
  for (int i = tid; i < kPrepWarps * E1; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int64_t per = ((S + kPrepWarps - 1) / kPrepWarps + 31) / 32 * 32;  // slots per warp, whole rounds
  const int64_t lo = min(S, (int64_t)warp * per), hi = min(S, lo + per);
  int32_t* h = hist + warp * E1;
  for (int64_t b = lo; b < hi; b += 32) {
    const int64_t sl = b + lane;
    int key = -1;
    if (sl < hi) {
      const int id = s_ids[sl];
      key = (id >= 0 && id < E) ? id : E;
    }
    const unsigned m = __match_any_sync(0xffffffffu, key);
    if (key >= 0 && lane == __ffs(m) - 1) h[key] += __popc(m);
    __syncwarp();
  }
  __syncthreads();
  for (int e = tid; e < E1; e += blockDim.x) {  // exclusive scan of each column over the warps
    int run = 0;
    for (int w = 0; w < kPrepWarps; ++w) {
      const int v = hist[w * E1 + e];
      hist[w * E1 + e] = run;
      run += v;
    }
    tot[e] = run;
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    const int t = (tot[e] + BM - 1) / BM;
    poff[e + 1] = t * BM;
    tcum[e + 1] = t;
  }
  if (tid == 0) {
    poff[0] = 0;
    tcum[0] = 0;
  }
  __syncthreads();
  smem_inclusive_scan<int32_t>(poff + 1, E, warp_sums);
  smem_inclusive_scan<int32_t>(tcum + 1, E, warp_sums);
  for (int e = lane; e < E; e += 32) h[e] += poff[e];  // this warp's first padded row per expert
  __syncwarp();
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int64_t b = lo; b < hi; b += 32) {
    const int64_t sl = b + lane;
    int key = -1;
    if (sl < hi) {
      const int id = s_ids[sl];
      key = (id >= 0 && id < E) ? id : E;
    }
    const unsigned m = __match_any_sync(0xffffffffu, key);
    if (key >= 0 && key < E) s_pos[sl] = h[key] + __popc(m & lt_mask);
    else if (key == E) s_pos[sl] = -1;
    __syncwarp();
    if (key >= 0 && key < E && lane == __ffs(m) - 1) h[key] += __popc(m);
    __syncwarp();
  }
  __syncthreads();

  if (blockIdx.x == 0) {
    for (int e = tid; e < E; e += blockDim.x) gs[e] = tot[e];
    for (int e = tid; e <= E; e += blockDim.x) {
      poff_out[e] = poff[e];
      table[TileTable::cum_off() + e] = tcum[e];
    }
    if (tid == 0) {
      table[0] = tcum[E];
      table[1] = poff[E];
      table[2] = tot[E];
      table[3] = 0;
    }
    const int ntiles = tcum[E];
    for (int i = tid; i < ntiles && i < max_tiles; i += blockDim.x) {
      int a = 0, z = E - 1;  // expert with tcum[a] <= i < tcum[a + 1]
      while (a < z) {
        const int mid = (a + z + 1) >> 1;
        if (tcum[mid] <= i) a = mid;
        else z = mid - 1;
      }
      const int j = i - tcum[a];
      table[TileTable::start_off(E) + i] = poff[a] + j * BM;
      table[TileTable::count_off(E, max_tiles) + i] = min(BM, tot[a] - j * BM);
    }
    for (int64_t sl = tid; sl < S; sl += blockDim.x) {
      const int pos = s_pos[sl];
      slot_pos[sl] = pos;
      if (pos >= 0) sorted[pos] = (int32_t)sl;
    }
  }

  // gather (+ int8 quantisation) of this CTA's slots, one warp per slot
  for (int64_t sl = (int64_t)blockIdx.x * kPrepWarps + warp; sl < S; sl += (int64_t)gridDim.x * kPrepWarps) {
    const int pos = s_pos[sl];
    if (pos < 0) continue;
    const Tin* src = x + (sl / k) * H;
    if constexpr (QUANT) {
      int8_t* d = static_cast<int8_t*>(xp) + (int64_t)pos * H;
      float amax = 0.f;
      for (int64_t c = lane * 8; c < H; c += 256) {
        float v[8];
        load8(src + c, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      float scale, inv;
      row_scales(amax, scale, inv);
      for (int64_t c = lane * 8; c < H; c += 256) {
        float v[8];
        load8(src + c, v);
        *reinterpret_cast<uint2*>(d + c) = quant8(v, inv);
      }
      if (lane == 0) xs[pos] = scale;
    } else {
      Tin* d = static_cast<Tin*>(xp) + (int64_t)pos * H;
      for (int64_t c = lane * 8; c < H; c += 256) copy8(src + c, d + c);
    }
  }

  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  if (kvalid) {  // routed slots per token; a token with none gets a zero output row here
    const int64_t T = S / k;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + tid; t < T; t += stride) {
      int c = 0;
      for (int j = 0; j < k; ++j) {
        const int id = s_ids[t * k + j];
        c += (id >= 0 && id < E);
      }
      kvalid[t] = c;
      if (c == 0)
        for (int64_t col = 0; col < H; col += 8) zero8(y + t * H + col);
    }
  }
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + tid; i < zero_a16; i += stride) zero_a[i] = z;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + tid; i < zero_b16; i += stride) zero_b[i] = z;
}

}  // namespace

bool prep_small_fits(int64_t slots, int num_experts) {
  return slots > 0 && slots <= kPrepMaxSlots && num_experts <= 1024;
}

int prep_small(const int32_t* topk_ids, int64_t num_tokens, int top_k, int num_experts, int block_m,
               const void* x, int x_dtype, int64_t hidden, void* xp, bool quant, float* xs, int32_t* sorted_slots,
               int32_t* slot_pos, int32_t* group_sizes, int32_t* padded_offsets, int32_t* tile_table,
               void* zero_a, size_t zero_a_bytes, void* zero_b, size_t zero_b_bytes, int32_t* kvalid, void* y,
               cudaStream_t st) {
  const int64_t S = num_tokens * top_k;
  MOE_CHECK_ARG(prep_small_fits(S, num_experts), "prep_small: batch too large");
  MOE_CHECK_ARG(hidden % 8 == 0 && zero_a_bytes % 16 == 0 && zero_b_bytes % 16 == 0, "prep_small: bad sizes");
  const int64_t max_tiles = moe_align_capacity(S, num_experts, block_m) / block_m;
  const size_t smem = ((size_t)2 * S + (size_t)(kPrepWarps + 3) * (num_experts + 1)) * sizeof(int32_t);
  int64_t grid = ceil_div(S, kPrepWarps);
  const int64_t zero16 = (int64_t)((zero_a_bytes + zero_b_bytes) / 16);
  grid = std::max<int64_t>(grid, ceil_div(zero16, (int64_t)kPrepThreads * 4));
  grid = std::min<int64_t>(std::max<int64_t>(grid, 1), num_sms());
#define PREP(TT, Q)                                                                                                \
  do {                                                                                                             \
    auto kfn = prep_small_kernel<TT, Q>;                                                                           \
    if (smem > 48 * 1024) MOE_CUDA_TRY(cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
    MOE_CUDA_TRY(launch_kernel(kfn, dim3((unsigned)grid), dim3(kPrepThreads), smem, st, topk_ids, S, top_k,          \
                               num_experts, block_m, max_tiles, static_cast<const TT*>(x), hidden, xp, xs,         \
                               sorted_slots, slot_pos, group_sizes, padded_offsets, tile_table,                    \
                               static_cast<uint4*>(zero_a), (int64_t)(zero_a_bytes / 16),                          \
                               static_cast<uint4*>(zero_b), (int64_t)(zero_b_bytes / 16), kvalid,                  \
                               static_cast<TT*>(y)));                                                              \
  } while (0)
  if (x_dtype == MOE_BF16) {
    if (quant) PREP(__nv_bfloat16, true);
    else PREP(__nv_bfloat16, false);
  } else if (x_dtype == MOE_F16) {
    if (quant) PREP(__half, true);
    else PREP(__half, false);
  } else {
    MOE_CHECK_ARG(!quant, "prep_small: int8 quantisation takes bf16/fp16 rows");
    PREP(float, false);
  }
#undef PREP
  MOE_LAUNCH_CHECK("prep_small_kernel");
  return MOE_OK;
}

}  // namespace moe
