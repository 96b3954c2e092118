// Router of one token on one warp, shared by the stand-alone router kernel
// (moe_route.cu) and phase 0 of the one-launch decode kernel (moe_decode.cuh).
//
// The k largest of the token's E logits are chosen (softmax and sigmoid are
// monotonic, so they are the k largest scores), ties going to the lower
// expert id; lane l holds experts l, l + 32, ... in registers (PER per lane,
// E <= 32 * PER). Choice j (j < k <= min(E, 32)) comes back on lane j: its
// expert id and its weight — the softmax over all E experts or the sigmoid
// of the logit, divided by the sum of the k chosen scores when renormalize is
// set. Lanes j >= k return id -1 and weight 0.
//
// Each round of the selection is two warp reductions: the largest remaining
// logit as an order-preserving 32-bit key (__reduce_max_sync), then the lowest
// expert id holding it (__reduce_min_sync). -0 counts as +0 (they compare
// equal as floats); a NaN logit ranks below every number. The scores are
// computed after the selection, lane j for choice j, and summed over the
// warp by a butterfly (every lane gets the same sum).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <climits>

namespace moe {

template <typename T>
__device__ __forceinline__ float route_to_f32(T v) {
  if constexpr (sizeof(T) == 4) return v;
  else return static_cast<float>(v);
}

// Float -> unsigned key with the same order (for non-NaN values).
__device__ __forceinline__ uint32_t route_key(float f) {
  const uint32_t u = __float_as_uint(f == 0.f ? 0.f : f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float route_unkey(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// This lane's PER logits of one token row (experts past E read as -inf).
template <typename T, int PER>
__device__ __forceinline__ void route_load(const T* __restrict__ row, int E, int lane, float (&v)[PER]) {
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? route_to_f32(row[e]) : -INFINITY;
  }
}

// Selection for N tokens of one warp at once (their reduction chains
// interleave); token n's choice j comes back on lane j of out_id[n] / out_w[n].
template <int N, int PER>
__device__ __forceinline__ void route_select(const float (&v)[N][PER], int E, int k, int sigmoid, int renormalize,
                                             int lane, int (&out_id)[N], float (&out_w)[N]) {
  // softmax over all experts needs the maximum and the partition function
  float m[N], z[N];
#pragma unroll
  for (int n = 0; n < N; ++n) {
    m[n] = -INFINITY;
    z[n] = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) m[n] = fmaxf(m[n], v[n][i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int n = 0; n < N; ++n) m[n] = fmaxf(m[n], __shfl_xor_sync(0xffffffffu, m[n], o));
  if (!sigmoid && !renormalize) {
#pragma unroll
    for (int n = 0; n < N; ++n)
#pragma unroll
      for (int i = 0; i < PER; ++i)
        if (lane + 32 * i < E) z[n] += expf(v[n][i] - m[n]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int n = 0; n < N; ++n) z[n] += __shfl_xor_sync(0xffffffffu, z[n], o);
  }
  // key 0: not a candidate (past E, or already chosen); a NaN ranks lowest
  uint32_t key[N][PER];
#pragma unroll
  for (int n = 0; n < N; ++n)
#pragma unroll
    for (int i = 0; i < PER; ++i)
      key[n][i] = lane + 32 * i < E ? (v[n][i] != v[n][i] ? 1u : route_key(v[n][i])) : 0u;
  uint32_t my_key[N];
  int my_j[N];
#pragma unroll
  for (int n = 0; n < N; ++n) {
    my_key[n] = 0u;
    my_j[n] = -1;
  }
  for (int j = 0; j < k; ++j) {
    uint32_t best[N];
    int bidx[N];
#pragma unroll
    for (int n = 0; n < N; ++n) {
      best[n] = 0u;
#pragma unroll
      for (int i = 0; i < PER; ++i) best[n] = max(best[n], key[n][i]);
    }
#pragma unroll
    for (int n = 0; n < N; ++n) best[n] = __reduce_max_sync(0xffffffffu, best[n]);
#pragma unroll
    for (int n = 0; n < N; ++n) {
      int cand = INT_MAX;
#pragma unroll
      for (int i = PER - 1; i >= 0; --i)
        if (key[n][i] == best[n]) cand = lane + 32 * i;
      bidx[n] = cand;
    }
#pragma unroll
    for (int n = 0; n < N; ++n) bidx[n] = __reduce_min_sync(0xffffffffu, bidx[n]);
#pragma unroll
    for (int n = 0; n < N; ++n) {
#pragma unroll
      for (int i = 0; i < PER; ++i)
        if (lane + 32 * i == bidx[n]) key[n][i] = 0u;
      if (lane == j) {
        my_j[n] = bidx[n];
        my_key[n] = best[n];
      }
    }
  }
  // scores of the k choices, one per lane, and their sum over the warp
  float score[N], sum[N];
#pragma unroll
  for (int n = 0; n < N; ++n) {
    const float bv = route_unkey(my_key[n]);
    score[n] = lane < k ? (sigmoid ? 1.0f / (1.0f + expf(-bv)) : expf(bv - m[n])) : 0.f;
    sum[n] = score[n];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int n = 0; n < N; ++n) sum[n] += __shfl_xor_sync(0xffffffffu, sum[n], o);
#pragma unroll
  for (int n = 0; n < N; ++n) {
    float w = score[n];
    if (renormalize) w = w / sum[n];
    else if (!sigmoid) w = w / z[n];
    out_id[n] = lane < k ? my_j[n] : -1;
    out_w[n] = lane < k ? w : 0.f;
  }
}

template <typename T, int PER>
__device__ __forceinline__ void route_token(const T* __restrict__ row, int E, int k, int sigmoid, int renormalize,
                                            int lane, int& out_id, float& out_w) {
  float v[1][PER];
  int id[1];
  float w[1];
  route_load<T, PER>(row, E, lane, v[0]);
  route_select<1, PER>(v, E, k, sigmoid, renormalize, lane, id, w);
  out_id = id[0];
  out_w = w[0];
}

}  // namespace moe
