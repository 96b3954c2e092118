// Router of one token on one warp, shared by the stand-alone router kernel
// (moe_route.cu) and phase 0 of the one-launch decode kernel (moe_decode.cuh).
//
// The k largest of the token's E logits are chosen (softmax and sigmoid are
// monotonic, so they are the k largest scores), ties going to the lower
// expert id; lane l holds experts l, l + 32, ... in registers (PER per lane,
// E <= 32 * PER). Choice j (j < k <= 32) comes back on lane j: its expert id
// and its weight — the softmax over all E experts or the sigmoid of the
// logit, divided by the sum of the k chosen scores when renormalize is set.
// Lanes j >= k return id -1 and weight 0.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace moe {

template <typename T>
__device__ __forceinline__ float route_to_f32(T v) {
  if constexpr (sizeof(T) == 4) return v;
  else return static_cast<float>(v);
}

template <typename T, int PER>
__device__ __forceinline__ void route_token(const T* __restrict__ row, int E, int k, int sigmoid, int renormalize,
                                            int lane, int& out_id, float& out_w) {
  float v[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? route_to_f32(row[e]) : -INFINITY;
  }
  // softmax over all experts needs the maximum and the partition function
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) m = fmaxf(m, v[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float z = 0.f;
  if (!sigmoid && !renormalize) {
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane + 32 * i < E) z += expf(v[i] - m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
  }
  unsigned taken = 0u;  // bit i: this lane's expert lane + 32 i already chosen
  float sel_sum = 0.f, my_score = 0.f;
  int my_j = -1;
  for (int j = 0; j < k; ++j) {
    float best = -INFINITY;
    int bidx = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !(taken >> i & 1u) && (v[i] > best || (v[i] == best && e < bidx))) {
        best = v[i];
        bidx = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
      if (ob > best || (ob == best && oi < bidx)) {
        best = ob;
        bidx = oi;
      }
    }
    if ((bidx & 31) == lane) taken |= 1u << (bidx >> 5);
    const float score = sigmoid ? 1.0f / (1.0f + expf(-best)) : expf(best - m);
    sel_sum += score;
    if (lane == j) {
      my_j = bidx;
      my_score = score;
    }
  }
  float w = 0.f;
  if (lane < k) {
    w = my_score;
    if (renormalize) w = w / sel_sum;
    else if (!sigmoid) w = w / z;
  }
  out_id = lane < k ? my_j : -1;
  out_w = w;
}

}  // namespace moe
