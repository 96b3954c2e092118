// CTA-wide prefix scans shared by the routing / schedule kernels.
#pragma once
#include <cstdint>

namespace moe {

// Inclusive scan of one value per thread across the CTA (<= 1024 threads).
template <typename T>
__device__ __forceinline__ T block_inclusive_scan(T v, T* warp_sums) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  if (lane == 31) warp_sums[warp] = v;
  __syncthreads();
  if (warp == 0) {
    T w = (lane < (int)(blockDim.x >> 5)) ? warp_sums[lane] : T(0);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      T n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    warp_sums[lane] = w;
  }
  __syncthreads();
  if (warp > 0) v += warp_sums[warp - 1];
  __syncthreads();
  return v;
}

// In-place inclusive scan of a[0..n) held in shared memory (one CTA).
template <typename T>
__device__ __forceinline__ void smem_inclusive_scan(T* a, int n, T* warp_sums) {
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int lo = min(n, (int)threadIdx.x * per), hi = min(n, lo + per);
  T local = 0;
  for (int i = lo; i < hi; ++i) local += a[i];
  T incl = block_inclusive_scan<T>(local, warp_sums);
  T run = incl - local;
  for (int i = lo; i < hi; ++i) {
    run += a[i];
    a[i] = run;
  }
  __syncthreads();
}

}  // namespace moe
