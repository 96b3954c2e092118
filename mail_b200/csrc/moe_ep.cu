// Expert parallelism over NVLink peer memory.
//
// Rank r owns experts [r*EL, (r+1)*EL). Every rank allocates, once, an
// IPC-shareable receive buffer that is laid out exactly like the padded,
// expert-sorted GEMM input of its local experts, plus a row-metadata array
// and a return buffer. One forward of the layer is then:
//
//   moe_align (block_m = 1)   this rank's slots sorted by global expert
//   all-gather of counts      [W, E] slot counts (NCCL, stream-ordered)
//   moe_ep_plan               where each of this rank's expert segments lands
//                             in its owner's buffer; this rank's local tile
//                             table; -1 metadata for its padding rows
//   moe_ep_dispatch           gather (+ int8 quant) of x rows, stored straight
//                             into the owners' receive buffers over NVLink
//   barrier                   (stream-ordered)
//   moe_ep_expert_pass        gate_up GEMM + SwiGLU -> down GEMM whose epilogue
//                             stores every output row straight into the return
//                             buffer of the rank that sent it
//   barrier
//   moe_combine_rows          weighted sum of the k returned rows per token
//
// No data moves through NCCL and no step needs a host synchronisation. The
// receive layout for destination d: its local expert el occupies padded rows
// [P_d(el), P_d(el) + pad128(N_el)), N_el = sum_s C[s][d*EL+el], and source
// s's rows of that expert start at P_d(el) + sum_{s'<s} C[s'][d*EL+el], in
// the source's stable slot order.
#include <cstring>

#include "common.cuh"
#include "scan.cuh"

namespace moe {
namespace {

constexpr int kPlanThreads = 1024;

__global__ void __launch_bounds__(kPlanThreads) ep_plan_kernel(
    const int32_t* __restrict__ counts_all, int W, int r, int E, int EL, int BM, int32_t* __restrict__ dest_base,
    int32_t* __restrict__ table, int64_t max_tiles, int32_t* __restrict__ meta_local, int64_t recv_cap,
    const int32_t* __restrict__ slot_pos, int64_t S, int32_t* __restrict__ ret_pos) {
  pdl_begin();
  extern __shared__ int32_t sm[];
  int32_t* pad = sm;       // [E]    padded totals, then their inclusive prefix
  int32_t* tcum = sm + E;  // [EL+1] tiles of this rank's local experts, prefix
  __shared__ int32_t warp_sums[32];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int tot = 0;
    for (int s = 0; s < W; ++s) tot += counts_all[(int64_t)s * E + e];
    pad[e] = (tot + BM - 1) / BM * BM;
  }
  __syncthreads();
  smem_inclusive_scan<int32_t>(pad, E, warp_sums);
  // where this rank's rows of expert e start in the owner's buffer
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int d = e / EL;
    const int block0 = d == 0 ? 0 : pad[d * EL - 1];
    const int excl = (e == 0 ? 0 : pad[e - 1]) - block0;
    int before = 0;
    for (int s = 0; s < r; ++s) before += counts_all[(int64_t)s * E + e];
    dest_base[e] = excl + before;
  }
  // this rank as a destination: tile table over its EL local experts
  const int block_r = r == 0 ? 0 : pad[r * EL - 1];
  for (int el = threadIdx.x; el < EL; el += blockDim.x) {
    const int e = r * EL + el;
    int tot = 0;
    for (int s = 0; s < W; ++s) tot += counts_all[(int64_t)s * E + e];
    tcum[el + 1] = (tot + BM - 1) / BM;
  }
  if (threadIdx.x == 0) tcum[0] = 0;
  __syncthreads();
  smem_inclusive_scan<int32_t>(tcum + 1, EL, warp_sums);
  const int total_rows = pad[r * EL + EL - 1] - block_r;
  int ntiles = tcum[EL];
  if ((int64_t)total_rows > recv_cap) ntiles = 0;  // cannot happen when sized by the worst case
  if (threadIdx.x == 0) {
    table[0] = ntiles;
    table[1] = total_rows;
    table[2] = (int64_t)total_rows > recv_cap ? 1 : 0;
    table[3] = 0;
  }
  for (int el = threadIdx.x; el <= EL; el += blockDim.x) table[TileTable::cum_off() + el] = ntiles ? tcum[el] : 0;
  for (int i = threadIdx.x; i < ntiles && i < max_tiles; i += blockDim.x) {
    int lo = 0, hi = EL - 1;  // local expert with tcum[el] <= i < tcum[el+1]
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tcum[mid] <= i) lo = mid;
      else hi = mid - 1;
    }
    const int el = lo, e = r * EL + el;
    int tot = 0;
    for (int s = 0; s < W; ++s) tot += counts_all[(int64_t)s * E + e];
    const int j = i - tcum[el];
    const int start = (e == 0 ? 0 : pad[e - 1]) - block_r + j * BM;
    const int cnt = min(BM, tot - j * BM);
    table[TileTable::start_off(EL) + i] = start;
    table[TileTable::count_off(EL, max_tiles) + i] = cnt;
    for (int rr = cnt; rr < BM; ++rr) meta_local[start + rr] = -1;
  }
  for (int64_t s = threadIdx.x; s < S; s += blockDim.x) ret_pos[s] = slot_pos[s] >= 0 ? (int32_t)s : -1;
}

__device__ __forceinline__ void ld8f(const __nv_bfloat16* p, float (&v)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void ld8f(const __half* p, float (&v)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// One warp per sorted slot: its token row goes to the owner's receive buffer
// (16-byte peer stores over NVLink), with the row's (source rank, slot) tag.
template <typename Tin, bool QUANT>
__global__ void __launch_bounds__(256) ep_dispatch_kernel(
    const Tin* __restrict__ x, int64_t H, int top_k, const int32_t* __restrict__ ids,
    const int32_t* __restrict__ sorted_slots, const int32_t* __restrict__ seg_start,
    const int32_t* __restrict__ dest_base, const int32_t* __restrict__ n_valid_dev, int64_t max_rows, int EL,
    int rank, int64_t recv_cap, void* const* __restrict__ peer_x, float* const* __restrict__ peer_scale,
    int32_t* const* __restrict__ peer_meta, int* __restrict__ err) {
  pdl_begin();
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t limit = min(max_rows, (int64_t)*n_valid_dev);
  for (int64_t p = warp; p < limit; p += nwarps) {
    const int32_t slot = sorted_slots[p];
    const int e = ids[slot];
    const int d = e / EL;
    const int64_t row = (int64_t)dest_base[e] + (p - seg_start[e]);
    if (row < 0 || row >= recv_cap) {
      if (lane == 0 && err) atomicExch(err, 1);
      continue;
    }
    const Tin* src = x + (int64_t)(slot / top_k) * H;
    if constexpr (QUANT) {
      float amax = 0.f;
      for (int64_t c = lane * 8; c < H; c += 256) {
        float v[8];
        ld8f(src + c, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float scale = __fdiv_rn(amax, 127.0f);
      const float inv = amax > 0.f ? __fdiv_rn(127.0f, amax) : 0.f;
      int8_t* dst = static_cast<int8_t*>(peer_x[d]) + row * H;
      for (int64_t c = lane * 8; c < H; c += 256) {
        float v[8];
        ld8f(src + c, v);
        uint32_t w[2] = {0u, 0u};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          int q = __float2int_rn(__fmul_rn(v[i], inv));
          q = max(-127, min(127, q));
          w[i >> 2] |= (uint32_t)(q & 0xff) << (8 * (i & 3));
        }
        *reinterpret_cast<uint2*>(dst + c) = make_uint2(w[0], w[1]);
      }
      if (lane == 0) peer_scale[d][row] = scale;
    } else {
      Tin* dst = static_cast<Tin*>(peer_x[d]) + row * H;
      for (int64_t c = lane * 8; c < H; c += 256)
        *reinterpret_cast<uint4*>(dst + c) = *reinterpret_cast<const uint4*>(src + c);
    }
    if (lane == 0) peer_meta[d][row] = (rank << 24) | slot;
  }
  __threadfence_system();
}

struct EpPassWs {
  size_t h, hq, hs, bytes;
};
EpPassWs ep_pass_ws(int64_t recv_cap, int64_t I, int x_dtype) {
  EpPassWs w;
  const bool q = x_dtype == MOE_I8;
  const int h_dtype = q ? MOE_BF16 : x_dtype;
  size_t off = 0;
  w.h = off;
  off = align_up(off + (size_t)recv_cap * I * dtype_size(h_dtype), 256);
  w.hq = off;
  off = align_up(off + (q ? (size_t)recv_cap * I : 0), 256);
  w.hs = off;
  off = align_up(off + (q ? (size_t)recv_cap * sizeof(float) : 0), 256);
  w.bytes = off;
  return w;
}

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" int moe_ipc_malloc(size_t bytes, void** ptr, void* handle) {
  MOE_CHECK_ARG(ptr && handle && bytes > 0, "moe_ipc_malloc: bad arguments");
  void* p = nullptr;
  MOE_CUDA_TRY(cudaMalloc(&p, bytes));
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return set_error(MOE_ERR_CUDA, "cudaIpcGetMemHandle failed: %s", cudaGetErrorString(e));
  }
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return MOE_OK;
}

extern "C" int moe_ipc_open(const void* handle, void** ptr) {
  MOE_CHECK_ARG(ptr && handle, "moe_ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  MOE_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return MOE_OK;
}

extern "C" int moe_ipc_close(void* ptr) {
  MOE_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return MOE_OK;
}

extern "C" int moe_ipc_free(void* ptr) {
  MOE_CUDA_TRY(cudaFree(ptr));
  return MOE_OK;
}

extern "C" int moe_ep_plan(const int32_t* counts_all, int world, int rank, int num_experts, const int32_t* slot_pos,
                           int64_t num_slots, int32_t* dest_base, int32_t* tile_table, int64_t max_tiles,
                           int32_t* recv_meta, int64_t recv_cap, int32_t* ret_pos, void* stream) {
  MOE_CHECK_ARG(world > 0 && world <= 128 && rank >= 0 && rank < world, "moe_ep_plan: bad world/rank");
  MOE_CHECK_ARG(num_experts > 0 && num_experts % world == 0 && num_experts <= 4096,
                "moe_ep_plan: num_experts must be a multiple of the world size (<= 4096)");
  MOE_CHECK_ARG(counts_all && dest_base && tile_table && recv_meta && (num_slots == 0 || (slot_pos && ret_pos)),
                "moe_ep_plan: NULL pointer");
  MOE_CHECK_ARG(recv_cap > 0 && recv_cap < (int64_t(1) << 31) && max_tiles >= recv_cap / kBlockM,
                "moe_ep_plan: bad receive capacity / max_tiles");
  const int EL = num_experts / world;
  const size_t smem = (size_t)(num_experts + EL + 1) * sizeof(int32_t);
  if (smem > 48 * 1024)
    MOE_CUDA_TRY(cudaFuncSetAttribute(ep_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  MOE_CUDA_TRY(launch_kernel(ep_plan_kernel, dim3(1), dim3(kPlanThreads), smem, as_stream(stream),
                             counts_all, world, rank, num_experts, EL, kBlockM, dest_base, tile_table,
                             max_tiles, recv_meta, recv_cap, slot_pos, num_slots, ret_pos));
  MOE_LAUNCH_CHECK("ep_plan_kernel");
  return MOE_OK;
}

extern "C" int moe_ep_dispatch(const void* x, int x_dtype, int64_t hidden, int top_k, const int32_t* topk_ids,
                               const int32_t* sorted_slots, const int32_t* seg_start, const int32_t* dest_base,
                               const int32_t* n_valid_dev, int64_t max_rows, int world, int rank,
                               int experts_per_rank, int64_t recv_cap, void* const* peer_x, int recv_dtype,
                               float* const* peer_scale, int32_t* const* peer_meta, int* err, void* stream) {
  MOE_CHECK_ARG(x && topk_ids && sorted_slots && seg_start && dest_base && n_valid_dev && peer_x && peer_meta,
                "moe_ep_dispatch: NULL pointer");
  MOE_CHECK_ARG(hidden > 0 && hidden % 8 == 0, "moe_ep_dispatch: hidden must be a positive multiple of 8");
  MOE_CHECK_ARG(world > 0 && rank >= 0 && rank < world && rank < 128 && experts_per_rank > 0,
                "moe_ep_dispatch: bad world/rank");
  MOE_CHECK_ARG(recv_cap > 0 && max_rows >= 0 && top_k > 0, "moe_ep_dispatch: bad sizes");
  if (max_rows == 0) return MOE_OK;
  int64_t blocks = ceil_div(max_rows, 8);
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  cudaStream_t st = as_stream(stream);
#define DISPATCH(TI, Q)                                                                                   \
  MOE_CUDA_TRY(launch_kernel(ep_dispatch_kernel<TI, Q>, dim3((unsigned)blocks), dim3(256), 0, st,         \
                             static_cast<const TI*>(x), hidden, top_k, topk_ids, sorted_slots, seg_start, \
                             dest_base, n_valid_dev, max_rows, experts_per_rank, rank, recv_cap, peer_x,  \
                             peer_scale, peer_meta, err))
  if (recv_dtype == MOE_I8) {
    MOE_CHECK_ARG(peer_scale != nullptr, "moe_ep_dispatch: int8 receive buffers need scales");
    if (x_dtype == MOE_BF16) DISPATCH(__nv_bfloat16, true);
    else if (x_dtype == MOE_F16) DISPATCH(__half, true);
    else return set_error(MOE_ERR_UNSUPPORTED, "moe_ep_dispatch: int8 dispatch takes bf16/fp16 rows");
  } else {
    MOE_CHECK_ARG(recv_dtype == x_dtype, "moe_ep_dispatch: receive dtype must equal x dtype (or int8)");
    if (x_dtype == MOE_BF16) DISPATCH(__nv_bfloat16, false);
    else if (x_dtype == MOE_F16) DISPATCH(__half, false);
    else return set_error(MOE_ERR_UNSUPPORTED, "moe_ep_dispatch: dtype %d not supported", x_dtype);
  }
#undef DISPATCH
  MOE_LAUNCH_CHECK("ep_dispatch_kernel");
  return MOE_OK;
}

extern "C" size_t moe_ep_expert_pass_workspace_size(int64_t recv_cap, int64_t inter, int x_dtype) {
  if (recv_cap <= 0 || inter <= 0 || dtype_size(x_dtype) == 0) return 0;
  return ep_pass_ws(recv_cap, inter, x_dtype).bytes;
}

extern "C" int moe_ep_expert_pass(const void* recv_x, int x_dtype, const float* recv_scale, int64_t recv_cap,
                                  int64_t hidden, const void* w13, const void* w2, int experts_per_rank,
                                  int64_t inter, const float* w13_scale, const float* w2_scale,
                                  const int32_t* tile_table, const int32_t* recv_meta, void* const* peer_ret,
                                  int world, int64_t ret_rows, int out_dtype, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  MOE_CHECK_ARG(x_dtype == MOE_BF16 || x_dtype == MOE_F16 || x_dtype == MOE_I8,
                "moe_ep_expert_pass: receive dtype must be bf16, fp16 or int8");
  MOE_CHECK_ARG(recv_cap > 0 && recv_cap % kBlockM == 0, "moe_ep_expert_pass: capacity must be whole tiles");
  MOE_CHECK_ARG(recv_x && w13 && w2 && tile_table && recv_meta && peer_ret, "moe_ep_expert_pass: NULL pointer");
  const bool q = x_dtype == MOE_I8;
  if (q) MOE_CHECK_ARG(recv_scale && w13_scale && w2_scale, "moe_ep_expert_pass: int8 needs scales");
  const int h_dtype = q ? MOE_BF16 : x_dtype;
  const EpPassWs w = ep_pass_ws(recv_cap, inter, x_dtype);
  if (workspace_bytes < w.bytes || !workspace)
    return set_error(MOE_ERR_WORKSPACE, "moe_ep_expert_pass: workspace %zu < %zu bytes", workspace_bytes, w.bytes);
  char* ws = static_cast<char*>(workspace);
  const int64_t max_tiles = recv_cap / kBlockM;
  cudaStream_t st = as_stream(stream);
  MOE_TRY(record_stage(MOE_STAGE_ENTRY, st));
  MOE_TRY(record_stage(MOE_STAGE_ROUTED, st));
  MOE_TRY(record_stage(MOE_STAGE_GATHERED, st));
  void* h = ws + w.h;
  MOE_TRY(moe_gemm1_swiglu(recv_x, x_dtype, recv_cap, hidden, w13, experts_per_rank, inter, recv_scale, w13_scale,
                           tile_table, max_tiles, h, h_dtype, stream));
  MOE_TRY(record_stage(MOE_STAGE_GEMM1, st));
  const void* a2 = h;
  float* hs = nullptr;
  if (q) {
    int8_t* hq = reinterpret_cast<int8_t*>(ws + w.hq);
    hs = reinterpret_cast<float*>(ws + w.hs);
    MOE_TRY(moe_quant_rows(h, h_dtype, recv_cap, inter, tile_table + 1, hq, hs, stream));
    a2 = hq;
  }
  MOE_TRY(record_stage(MOE_STAGE_PRE_GEMM2, st));
  MOE_TRY(gemm2_scatter_peer(a2, q ? MOE_I8 : h_dtype, recv_cap, inter, w2, experts_per_rank, hidden, hs, w2_scale,
                             tile_table, max_tiles, recv_meta, peer_ret, world, ret_rows, out_dtype, st));
  MOE_TRY(record_stage(MOE_STAGE_GEMM2, st));
  MOE_TRY(record_stage(MOE_STAGE_DONE, st));
  return MOE_OK;
}
