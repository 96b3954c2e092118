// Row-wise HBM-bound kernels around the grouped GEMMs: the permuting gather
// (optionally fused with per-token int8 quantisation), the deterministic
// weighted combine, and the fp32 -> output-dtype conversion.
//
// All of them move whole rows with 16-byte vector accesses, one warp per row,
// grid-stride over rows with the grid sized as a multiple of the SM count.
#include "common.cuh"
#include "rows.cuh"

namespace moe {
namespace {
using namespace rows;

template <typename Tin, typename Tout>
__global__ void __launch_bounds__(256) gather_rows_kernel(const Tin* __restrict__ src, int64_t cols,
                                                          const int32_t* __restrict__ slots, int top_k,
                                                          int64_t rows, const int32_t* __restrict__ rows_dev,
                                                          Tout* __restrict__ dst, float* __restrict__ dst_scale,
                                                          int zero_pad) {
  pdl_begin();
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  int64_t limit = rows;
  if (rows_dev) limit = min(limit, (int64_t)*rows_dev);
  for (int64_t p = warp; p < limit; p += nwarps) {
    const int64_t slot = slots ? (int64_t)slots[p] : p;
    Tout* d = dst + p * cols;
    if (slot < 0) {
      if (!zero_pad) continue;
      for (int64_t c = lane * 8; c < cols; c += 256) zero8(d + c);
      if constexpr (sizeof(Tout) == 1)
        if (lane == 0 && dst_scale) dst_scale[p] = 0.f;
      continue;
    }
    const Tin* s = src + (slot / top_k) * cols;
    if constexpr (sizeof(Tout) == 1) {
      float amax = 0.f;
      for (int64_t c = lane * 8; c < cols; c += 256) {
        float v[8];
        load8(s + c, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      float scale, inv;
      row_scales(amax, scale, inv);
      for (int64_t c = lane * 8; c < cols; c += 256) {
        float v[8];
        load8(s + c, v);
        *reinterpret_cast<uint2*>(d + c) = quant8(v, inv);
      }
      if (lane == 0 && dst_scale) dst_scale[p] = scale;
    } else {
      for (int64_t c = lane * 8; c < cols; c += 256) copy8(s + c, d + c);
    }
  }
}

// Gather + per-token int8 quantisation with RT threads per row (a 128-thread
// CTA handles 128 / RT rows at a time): each thread keeps up to kQuantVecs
// 8-element vectors of its row in registers, so the row is read once with 8
// independent 16-byte loads in flight per thread, reduced to its absmax
// across the RT threads, then quantised from registers. RT is chosen so the
// threads are full: 32 for rows <= 2048 columns, 64 for <= 4096, else 128
// (rows up to 8192 columns). A padding row (slot < 0) quantises zeros, or is
// skipped when zero_pad is 0.
constexpr int kQuantVecs = 8;
constexpr int kQuantThreads = 128;
constexpr int64_t kQuantMaxCols = (int64_t)kQuantThreads * 8 * kQuantVecs;

template <typename Tin, int RT>
__global__ void __launch_bounds__(kQuantThreads) gather_quant_kernel(const Tin* __restrict__ src, int64_t cols,
                                                                     const int32_t* __restrict__ slots, int top_k,
                                                                     int64_t rows,
                                                                     const int32_t* __restrict__ rows_dev,
                                                                     int8_t* __restrict__ dst,
                                                                     float* __restrict__ dst_scale, int zero_pad) {
  pdl_begin();
  constexpr int kRowsPerPass = kQuantThreads / RT;
  constexpr int kWarpsPerRow = RT / 32;
  __shared__ float red[kQuantThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = tid / RT, gt = tid % RT;
  int64_t limit = rows;
  if (rows_dev) limit = min(limit, (int64_t)*rows_dev);
  for (int64_t base = (int64_t)blockIdx.x * kRowsPerPass; base < limit; base += (int64_t)gridDim.x * kRowsPerPass) {
    const int64_t p = base + grp;
    const bool active = p < limit;
    const int64_t slot = active ? (slots ? (int64_t)slots[p] : p) : -1;
    const Tin* s = slot >= 0 ? src + (slot / top_k) * cols : nullptr;
    float v[kQuantVecs][8];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < kQuantVecs; ++i) {
      const int64_t c = ((int64_t)i * RT + gt) * 8;
      if (s && c < cols) {
        load8(s + c, v[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if constexpr (kWarpsPerRow > 1) {
      if (lane == 0) red[warp] = amax;
      __syncthreads();
      const int w0 = grp * kWarpsPerRow;
      amax = red[w0];
#pragma unroll
      for (int w = 1; w < kWarpsPerRow; ++w) amax = fmaxf(amax, red[w0 + w]);
      __syncthreads();
    }
    float scale, inv;
    row_scales(amax, scale, inv);
    if (active && (slot >= 0 || zero_pad)) {
      int8_t* d = dst + p * cols;
#pragma unroll
      for (int i = 0; i < kQuantVecs; ++i) {
        const int64_t c = ((int64_t)i * RT + gt) * 8;
        if (c < cols) *reinterpret_cast<uint2*>(d + c) = quant8(v[i], inv);
      }
      if (gt == 0 && dst_scale) dst_scale[p] = scale;
    }
  }
}

// Token-order scatter of the routed rows, the inverse of the gather: each
// token's row is read once (RT threads per row, kept in registers), quantised
// once when Tout is int8 (the quantisation is per token, so all k copies
// share it), and stored to each of its k padded rows slot_pos[t * k + j]
// (skipped where < 0). Reads T x H instead of the gather's T x k x H, which
// comes from DRAM once the activations outgrow the L2.
template <typename Tin, typename Tout, int RT>
__global__ void __launch_bounds__(kQuantThreads) scatter_rows_kernel(const Tin* __restrict__ src, int64_t cols,
                                                                     const int32_t* __restrict__ slot_pos,
                                                                     int top_k, int64_t T,
                                                                     Tout* __restrict__ dst,
                                                                     float* __restrict__ dst_scale) {
  pdl_begin();
  constexpr bool QUANT = sizeof(Tout) == 1;
  constexpr int kRowsPerPass = kQuantThreads / RT;
  constexpr int kWarpsPerRow = RT / 32;
  __shared__ float red[kQuantThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = tid / RT, gt = tid % RT;
  for (int64_t base = (int64_t)blockIdx.x * kRowsPerPass; base < T; base += (int64_t)gridDim.x * kRowsPerPass) {
    const int64_t t = base + grp;
    const bool active = t < T;
    const Tin* s = active ? src + t * cols : nullptr;
    float v[kQuantVecs][8];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < kQuantVecs; ++i) {
      const int64_t c = ((int64_t)i * RT + gt) * 8;
      if (s && c < cols) {
        load8(s + c, v[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
      }
    }
    float scale = 0.f, inv = 0.f;
    if constexpr (QUANT) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if constexpr (kWarpsPerRow > 1) {
        if (lane == 0) red[warp] = amax;
        __syncthreads();
        const int w0 = grp * kWarpsPerRow;
        amax = red[w0];
#pragma unroll
        for (int w = 1; w < kWarpsPerRow; ++w) amax = fmaxf(amax, red[w0 + w]);
        __syncthreads();
      }
      row_scales(amax, scale, inv);
    }
    if (!active) continue;
    for (int j = 0; j < top_k; ++j) {
      const int32_t pos = slot_pos[t * top_k + j];
      if (pos < 0) continue;
      Tout* d = dst + (int64_t)pos * cols;
#pragma unroll
      for (int i = 0; i < kQuantVecs; ++i) {
        const int64_t c = ((int64_t)i * RT + gt) * 8;
        if (c >= cols) continue;
        if constexpr (QUANT) *reinterpret_cast<uint2*>(d + c) = quant8(v[i], inv);
        else store8(d + c, v[i]);
      }
      if (QUANT && gt == 0 && dst_scale) dst_scale[pos] = scale;
    }
  }
}

template <typename To, typename Tacc>
__global__ void __launch_bounds__(256) combine_rows_kernel(const To* __restrict__ o, int64_t hidden,
                                                           const int32_t* __restrict__ slot_pos,
                                                           const float* __restrict__ w, int64_t T, int k,
                                                           Tacc* __restrict__ y) {
  pdl_begin();
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t t = warp; t < T; t += nwarps) {
    for (int64_t c = lane * 8; c < hidden; c += 256) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int j = 0; j < k; ++j) {
        const int32_t pos = slot_pos[t * k + j];
        if (pos < 0) continue;
        const float wj = w[t * k + j];
        float v[8];
        load8(o + (int64_t)pos * hidden + c, v);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = fmaf(wj, v[i], acc[i]);
      }
      store8(y + t * hidden + c, acc);
    }
  }
}

template <typename Tout>
__global__ void __launch_bounds__(256) convert_f32_kernel(const float* __restrict__ src, int64_t n8,
                                                          Tout* __restrict__ dst) {
  pdl_begin();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    float v[8];
    load8(src + i * 8, v);
    store8(dst + i * 8, v);
  }
}

unsigned row_grid(int64_t rows) {
  const int64_t per_block = 8;  // warps per 256-thread block
  int64_t blocks = ceil_div(rows, per_block);
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  return (unsigned)(blocks < 1 ? 1 : blocks);
}

// Zero fill of n16 16-byte words (a kernel rather than a memset so that it
// takes part in programmatic dependent launch).
__global__ void __launch_bounds__(256) zero16_kernel(uint4* __restrict__ dst, int64_t n16) {
  pdl_begin();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = make_uint4(0u, 0u, 0u, 0u);
}

}  // namespace

int zero_fill(void* dst, size_t bytes, cudaStream_t st) {
  if (bytes == 0) return MOE_OK;
  if ((uintptr_t)dst % 16 != 0 || bytes % 16 != 0) {  // not the case for the library's own buffers
    MOE_CUDA_TRY(cudaMemsetAsync(dst, 0, bytes, st));
    return MOE_OK;
  }
  const int64_t n16 = (int64_t)(bytes / 16);
  int64_t blocks = ceil_div(n16, 256 * 4);
  const int64_t cap = (int64_t)num_sms() * 8;
  if (blocks > cap) blocks = cap;
  MOE_CUDA_TRY(launch_kernel(zero16_kernel, dim3((unsigned)blocks), dim3(256), 0, st, static_cast<uint4*>(dst), n16));
  MOE_LAUNCH_CHECK("zero16_kernel");
  return MOE_OK;
}
}  // namespace moe

using namespace moe;

namespace moe {
bool scatter_rows_fits(int64_t cols) { return cols > 0 && cols % 8 == 0 && cols <= kQuantMaxCols; }

int scatter_rows(const void* src, int src_dtype, int64_t cols, const int32_t* slot_pos, int top_k, int64_t T,
                 void* dst, int dst_dtype, float* dst_scale, cudaStream_t st) {
  MOE_CHECK_ARG(src && dst && slot_pos, "scatter_rows: NULL pointer");
  MOE_CHECK_ARG(scatter_rows_fits(cols), "scatter_rows: cols %lld unsupported", (long long)cols);
  MOE_CHECK_ARG(((uintptr_t)src % 16 == 0) && ((uintptr_t)dst % 16 == 0), "scatter_rows: pointers must be 16-byte aligned");
  if (T == 0) return MOE_OK;
  const int rt = cols <= 2048 ? 32 : (cols <= 4096 ? 64 : 128);
  int64_t blocks = ceil_div(T, kQuantThreads / rt);
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
#define SCATTER(TI, TO, RT)                                                                                        \
  MOE_CUDA_TRY(launch_kernel(scatter_rows_kernel<TI, TO, RT>, dim3((unsigned)blocks), dim3(kQuantThreads), 0, st, \
                             static_cast<const TI*>(src), cols, slot_pos, top_k, T, static_cast<TO*>(dst),         \
                             dst_scale))
#define SCATTER_RT(TI, TO)           \
  if (rt == 32) SCATTER(TI, TO, 32);  \
  else if (rt == 64) SCATTER(TI, TO, 64); \
  else SCATTER(TI, TO, 128);
  if (dst_dtype == MOE_I8) {
    MOE_CHECK_ARG(dst_scale != nullptr, "scatter_rows: int8 output needs dst_scale");
    if (src_dtype == MOE_BF16) { SCATTER_RT(__nv_bfloat16, int8_t) }
    else if (src_dtype == MOE_F16) { SCATTER_RT(__half, int8_t) }
    else if (src_dtype == MOE_F32) { SCATTER_RT(float, int8_t) }
    else return set_error(MOE_ERR_UNSUPPORTED, "scatter_rows: dtype %d not supported", src_dtype);
  } else {
    MOE_CHECK_ARG(dst_dtype == src_dtype, "scatter_rows: output dtype must be int8 or the input's");
    if (src_dtype == MOE_BF16) { SCATTER_RT(__nv_bfloat16, __nv_bfloat16) }
    else if (src_dtype == MOE_F16) { SCATTER_RT(__half, __half) }
    else if (src_dtype == MOE_F32) { SCATTER_RT(float, float) }
    else return set_error(MOE_ERR_UNSUPPORTED, "scatter_rows: dtype %d not supported", src_dtype);
  }
#undef SCATTER_RT
#undef SCATTER
  MOE_LAUNCH_CHECK("scatter_rows_kernel");
  return MOE_OK;
}

// moe_gather_rows with a choice for padding rows (slot < 0): zero-filled
// (zero_pad), or left as they are. The fused top-k pass leaves them: the
// GEMMs compute padding rows but never store their results, so their content
// does not matter (at one token over 128 experts the rows are 99 % padding).
int gather_rows(const void* src, int src_dtype, int64_t cols, const int32_t* sorted_slots, int top_k, int64_t rows,
                const int32_t* rows_dev, void* dst, int dst_dtype, float* dst_scale, bool zero_pad, void* stream) {
  MOE_CHECK_ARG(src && dst, "moe_gather_rows: NULL src/dst");
  MOE_CHECK_ARG(cols > 0 && cols % 8 == 0, "moe_gather_rows: cols (%lld) must be a positive multiple of 8",
                (long long)cols);
  MOE_CHECK_ARG(top_k > 0 && rows >= 0, "moe_gather_rows: bad top_k/rows");
  MOE_CHECK_ARG(((uintptr_t)src % 16 == 0) && ((uintptr_t)dst % 16 == 0),
                "moe_gather_rows: pointers must be 16-byte aligned");
  if (rows == 0) return MOE_OK;
  cudaStream_t st = as_stream(stream);
  const unsigned grid = row_grid(rows);
#define GATHER(TI, TO)                                                                               \
  MOE_CUDA_TRY(launch_kernel(gather_rows_kernel<TI, TO>, dim3(grid), dim3(256), 0, st,               \
                             static_cast<const TI*>(src), cols, sorted_slots, top_k, rows, rows_dev, \
                             static_cast<TO*>(dst), dst_scale, (int)zero_pad))
  if (dst_dtype == src_dtype) {
    if (src_dtype == MOE_BF16) GATHER(__nv_bfloat16, __nv_bfloat16);
    else if (src_dtype == MOE_F16) GATHER(__half, __half);
    else if (src_dtype == MOE_F32) GATHER(float, float);
    else return set_error(MOE_ERR_UNSUPPORTED, "moe_gather_rows: dtype %d not supported", src_dtype);
  } else if (dst_dtype == MOE_I8) {
    MOE_CHECK_ARG(dst_scale != nullptr, "moe_gather_rows: int8 output needs dst_scale");
    if (cols <= kQuantMaxCols) {
      const int rt = cols <= 2048 ? 32 : (cols <= 4096 ? 64 : 128);
      int64_t blocks = ceil_div(rows, kQuantThreads / rt);
      const int64_t cap = (int64_t)num_sms() * 16;
      if (blocks > cap) blocks = cap;
#define GATHER_Q(TI, RT)                                                                                      \
  MOE_CUDA_TRY(launch_kernel(gather_quant_kernel<TI, RT>, dim3((unsigned)blocks), dim3(kQuantThreads), 0, st, \
                             static_cast<const TI*>(src), cols, sorted_slots, top_k, rows, rows_dev,          \
                             static_cast<int8_t*>(dst), dst_scale, (int)zero_pad))
#define GATHER_QT(TI)                  \
  if (rt == 32) GATHER_Q(TI, 32);      \
  else if (rt == 64) GATHER_Q(TI, 64); \
  else GATHER_Q(TI, 128);
      if (src_dtype == MOE_BF16) {
        GATHER_QT(__nv_bfloat16)
      } else if (src_dtype == MOE_F16) {
        GATHER_QT(__half)
      } else if (src_dtype == MOE_F32) {
        GATHER_QT(float)
      } else {
        return set_error(MOE_ERR_UNSUPPORTED, "moe_gather_rows: dtype %d not supported", src_dtype);
      }
#undef GATHER_QT
#undef GATHER_Q
      MOE_LAUNCH_CHECK("gather_quant_kernel");
      return MOE_OK;
    }
    if (src_dtype == MOE_BF16) GATHER(__nv_bfloat16, int8_t);
    else if (src_dtype == MOE_F16) GATHER(__half, int8_t);
    else if (src_dtype == MOE_F32) GATHER(float, int8_t);
    else return set_error(MOE_ERR_UNSUPPORTED, "moe_gather_rows: dtype %d not supported", src_dtype);
  } else {
    return set_error(MOE_ERR_UNSUPPORTED, "moe_gather_rows: %d -> %d not supported", src_dtype, dst_dtype);
  }
#undef GATHER
  MOE_LAUNCH_CHECK("gather_rows_kernel");
  return MOE_OK;
}
}  // namespace moe

extern "C" int moe_gather_rows(const void* src, int src_dtype, int64_t cols, const int32_t* sorted_slots,
                               int top_k, int64_t rows, const int32_t* rows_dev, void* dst, int dst_dtype,
                               float* dst_scale, void* stream) {
  return gather_rows(src, src_dtype, cols, sorted_slots, top_k, rows, rows_dev, dst, dst_dtype, dst_scale, true,
                     stream);
}

extern "C" int moe_quant_rows(const void* src, int src_dtype, int64_t rows, int64_t cols, const int32_t* rows_dev,
                              int8_t* dst, float* dst_scale, void* stream) {
  return moe_gather_rows(src, src_dtype, cols, nullptr, 1, rows, rows_dev, dst, MOE_I8, dst_scale, stream);
}

extern "C" int moe_combine_rows(const void* o, int o_dtype, int64_t hidden, const int32_t* slot_pos,
                                const float* topk_weights, int64_t num_tokens, int top_k, void* y, int y_dtype,
                                void* stream) {
  MOE_CHECK_ARG(o && slot_pos && topk_weights && y, "moe_combine_rows: NULL pointer");
  MOE_CHECK_ARG(hidden > 0 && hidden % 8 == 0, "moe_combine_rows: hidden must be a positive multiple of 8");
  MOE_CHECK_ARG(num_tokens >= 0 && top_k > 0, "moe_combine_rows: bad num_tokens/top_k");
  if (num_tokens == 0) return MOE_OK;
  cudaStream_t st = as_stream(stream);
  const unsigned grid = row_grid(num_tokens);
#define COMBINE(TO, TY)                                                                                    \
  MOE_CUDA_TRY(launch_kernel(combine_rows_kernel<TO, TY>, dim3(grid), dim3(256), 0, st,                    \
                             static_cast<const TO*>(o), hidden, slot_pos, topk_weights, num_tokens, top_k, \
                             static_cast<TY*>(y)))
  if (o_dtype == MOE_BF16 && y_dtype == MOE_BF16) COMBINE(__nv_bfloat16, __nv_bfloat16);
  else if (o_dtype == MOE_F16 && y_dtype == MOE_F16) COMBINE(__half, __half);
  else if (o_dtype == MOE_F32 && y_dtype == MOE_F32) COMBINE(float, float);
  else if (o_dtype == MOE_BF16 && y_dtype == MOE_F32) COMBINE(__nv_bfloat16, float);
  else return set_error(MOE_ERR_UNSUPPORTED, "moe_combine_rows: %d -> %d not supported", o_dtype, y_dtype);
#undef COMBINE
  MOE_LAUNCH_CHECK("combine_rows_kernel");
  return MOE_OK;
}

extern "C" int moe_convert_f32(const float* src, int64_t n, void* dst, int dst_dtype, void* stream) {
  MOE_CHECK_ARG(src && dst, "moe_convert_f32: NULL pointer");
  MOE_CHECK_ARG(n >= 0 && n % 8 == 0, "moe_convert_f32: n must be a multiple of 8");
  if (n == 0) return MOE_OK;
  cudaStream_t st = as_stream(stream);
  const int64_t n8 = n / 8;
  int64_t blocks = ceil_div(n8, 256);
  const int64_t cap = (int64_t)num_sms() * 8;
  if (blocks > cap) blocks = cap;
  if (dst_dtype == MOE_BF16)
    MOE_CUDA_TRY(launch_kernel(convert_f32_kernel<__nv_bfloat16>, dim3((unsigned)blocks), dim3(256), 0, st,
                               src, n8, static_cast<__nv_bfloat16*>(dst)));
  else if (dst_dtype == MOE_F16)
    MOE_CUDA_TRY(launch_kernel(convert_f32_kernel<__half>, dim3((unsigned)blocks), dim3(256), 0, st,
                               src, n8, static_cast<__half*>(dst)));
  else if (dst_dtype == MOE_F32)
    MOE_CUDA_TRY(launch_kernel(convert_f32_kernel<float>, dim3((unsigned)blocks), dim3(256), 0, st,
                               src, n8, static_cast<float*>(dst)));
  else
    return set_error(MOE_ERR_UNSUPPORTED, "moe_convert_f32: dtype %d not supported", dst_dtype);
  MOE_LAUNCH_CHECK("convert_f32_kernel");
  return MOE_OK;
}
