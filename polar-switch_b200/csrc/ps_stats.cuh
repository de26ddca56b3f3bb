// Per-matrix telemetry of orthogonalized updates in one pass over them: the
// numbers of NaN and infinite entries and the largest |x| over the entries
// that are not NaN. The reference's NormLog (training/diagnostics.py:161-165)
// takes these as three separate passes (isnan().sum, isinf().sum,
// abs().amax) over every update it records.
//
// Counts are exact in any order; the maximum is order-independent too, and is
// combined across blocks with an integer atomicMax on the bit pattern, which
// orders non-negative floats (infinity above every finite value) the way the
// floats are ordered.
#pragma once

#include "ps_norm.cuh"

namespace ps {

__device__ __forceinline__ void stats_add(float v, unsigned long long& nan, unsigned long long& inf,
                                          float& amax) {
  if (isnan(v)) {
    ++nan;  // fmaxf below would ignore it anyway
    return;
  }
  if (isinf(v)) ++inf;
  amax = fmaxf(amax, fabsf(v));
}

// Grid (blocks per matrix, matrices); matrix l is E contiguous elements at
// x + l * E. nan_count / inf_count / amax_bits must be zero before the launch.
template <typename T>
__global__ void __launch_bounds__(NORM_THREADS)
    ps_update_stats_kernel(const T* __restrict__ x, long long E,
                           unsigned long long* __restrict__ nan_count,
                           unsigned long long* __restrict__ inf_count,
                           unsigned int* __restrict__ amax_bits) {
  __shared__ unsigned long long s_nan[NORM_THREADS / 32], s_inf[NORM_THREADS / 32];
  __shared__ float s_max[NORM_THREADS / 32];
  const long long l = blockIdx.y;
  const T* xm = x + l * E;
  unsigned long long nan = 0, inf = 0;
  float amax = 0.f;
  const long long stride = static_cast<long long>(gridDim.x) * NORM_THREADS;
  const long long first = static_cast<long long>(blockIdx.x) * NORM_THREADS + threadIdx.x;
  long long tail = 0;
  if (is_aligned16(xm)) {
    const long long n8 = E / 8;
    for (long long v = first; v < n8; v += stride) {
      float f[8];
      load8(xm + v * 8, f);
#pragma unroll
      for (int k = 0; k < 8; ++k) stats_add(f[k], nan, inf, amax);
    }
    tail = n8 * 8;
  }
  for (long long e = tail + first; e < E; e += stride) stats_add(to_f32(xm[e]), nan, inf, amax);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    nan += __shfl_xor_sync(0xffffffffu, nan, o);
    inf += __shfl_xor_sync(0xffffffffu, inf, o);
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  }
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    s_nan[warp] = nan;
    s_inf[warp] = inf;
    s_max[warp] = amax;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < NORM_THREADS / 32; ++w) {
      nan += s_nan[w];
      inf += s_inf[w];
      amax = fmaxf(amax, s_max[w]);
    }
    if (nan) atomicAdd(nan_count + l, nan);
    if (inf) atomicAdd(inf_count + l, inf);
    atomicMax(amax_bits + l, __float_as_uint(amax));
  }
}

}  // namespace ps
