// Muon's step before the circuit (training/muon.py:63-74) for a bucket of
// same-shape matrices, in one pass over their gradients and momentum buffers:
//
//   m <- fl(fl(m * mu) + g)            buf.mul_(momentum).add_(grad)
//   d  = fl(g + mu * m)   (Nesterov)   grad.add(buf, alpha=momentum)
//      = m                (plain)
//   out[p] = cast(d)                   torch.stack(directions) [.bfloat16()]
//
// m and d are rounded to the parameters' dtype T exactly where torch rounds
// them (after the multiply, after the add, after `g + mu * m`, evaluated in
// FP32), then d is cast to the output dtype. The unfused sequence reads and
// writes each element of the momentum, the gradient, the direction and the
// stacked copy several times; here each is touched once.
#pragma once

#include <type_traits>

#include "ps_norm.cuh"

namespace ps {

constexpr int MUON_MAX_PARAMS = 64;

struct MuonDirectionArgs {
  const void* grad[MUON_MAX_PARAMS];
  void* mom[MUON_MAX_PARAMS];
  long long E;       // elements per matrix
  float mu;
  int nesterov;
};

template <typename T>
__device__ __forceinline__ float round_to(float v);
template <>
__device__ __forceinline__ float round_to<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float round_to<__nv_bfloat16>(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}
template <>
__device__ __forceinline__ float round_to<__half>(float v) {
  return __half2float(__float2half_rn(v));
}

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(v);
}

// The element-wise kernels below move 8 elements per thread and iteration
// (load8 of ps_norm.cuh, store8 here: 16-byte accesses, two for FP32) when
// every pointer is 16-byte aligned and a matrix holds a multiple of 8 elements.

// Rounds eight FP32 values to T's precision in place (round to nearest
// even), two per packed convert for the 16-bit types; the same values as
// round_to<T> on each.
template <typename T>
__device__ __forceinline__ void round8(float (&f)[8]) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 g = __bfloat1622float2(__floats2bfloat162_rn(f[2 * j], f[2 * j + 1]));
      f[2 * j] = g.x;
      f[2 * j + 1] = g.y;
    }
  } else if constexpr (std::is_same<T, __half>::value) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 g = __half22float2(__floats2half2_rn(f[2 * j], f[2 * j + 1]));
      f[2 * j] = g.x;
      f[2 * j + 1] = g.y;
    }
  }
}

// Stores f (values representable in T) as eight elements of T.
template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&f)[8]) {
  if constexpr (sizeof(T) == 4) {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const T lo = from_f32<T>(f[2 * j]), hi = from_f32<T>(f[2 * j + 1]);
      unsigned short l, h;
      memcpy(&l, &lo, 2);
      memcpy(&h, &hi, 2);
      w[j] = static_cast<uint32_t>(l) | (static_cast<uint32_t>(h) << 16);
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// grid (x: blocks over the elements, y: matrices of this launch); VEC = 8:
// eight elements per thread and iteration (aligned pointers, E % 8 == 0).
template <typename T, typename TO, int VEC>
__global__ void __launch_bounds__(NORM_THREADS)
    ps_muon_direction_kernel(const __grid_constant__ MuonDirectionArgs a, TO* __restrict__ out) {
  const int p = blockIdx.y;
  const T* g = static_cast<const T*>(a.grad[p]);
  T* m = static_cast<T*>(a.mom[p]);
  TO* o = out + static_cast<long long>(p) * a.E;
  const long long stride = static_cast<long long>(gridDim.x) * NORM_THREADS;
  const long long first = static_cast<long long>(blockIdx.x) * NORM_THREADS + threadIdx.x;
  if constexpr (VEC == 8) {
    for (long long v = first; v < a.E / 8; v += stride) {
      float gv[8], mv[8], m2[8], d[8];
      load8(g + 8 * v, gv);
      load8(m + 8 * v, mv);
#pragma unroll
      for (int j = 0; j < 8; ++j) m2[j] = __fmul_rn(mv[j], a.mu);
      round8<T>(m2);
#pragma unroll
      for (int j = 0; j < 8; ++j) m2[j] = __fadd_rn(m2[j], gv[j]);
      round8<T>(m2);
#pragma unroll
      for (int j = 0; j < 8; ++j) d[j] = a.nesterov ? __fmaf_rn(a.mu, m2[j], gv[j]) : m2[j];
      round8<T>(d);
      store8(m + 8 * v, m2);
      round8<TO>(d);
      store8(o + 8 * v, d);
    }
  } else {
    for (long long e = first; e < a.E; e += stride) {
      const float gv = to_f32(g[e]);
      const float m1 = round_to<T>(__fmul_rn(to_f32(m[e]), a.mu));
      const float m2 = round_to<T>(__fadd_rn(m1, gv));
      m[e] = from_f32<T>(m2);
      const float d = a.nesterov ? round_to<T>(__fmaf_rn(a.mu, m2, gv)) : m2;
      o[e] = from_f32<TO>(d);
    }
  }
}

// Muon's step after the circuit (training/muon.py:84-86) for a bucket:
//   p <- fl(fl(p * decay) + alpha * fl_T(u[i]))
// (p.mul_(1 - lr * wd); p.add_(u.to(p.dtype), alpha=-lr * factor)), with p of
// dtype T rounded where torch rounds it and u the circuit's stacked output.
struct MuonUpdateArgs {
  void* param[MUON_MAX_PARAMS];
  long long E;
  float decay, alpha;
};

template <typename T, typename TU, int VEC>
__global__ void __launch_bounds__(NORM_THREADS)
    ps_muon_update_kernel(const __grid_constant__ MuonUpdateArgs a, const TU* __restrict__ upd) {
  const int p = blockIdx.y;
  T* w = static_cast<T*>(a.param[p]);
  const TU* u = upd + static_cast<long long>(p) * a.E;
  const long long stride = static_cast<long long>(gridDim.x) * NORM_THREADS;
  const long long first = static_cast<long long>(blockIdx.x) * NORM_THREADS + threadIdx.x;
  if constexpr (VEC == 8) {
    for (long long v = first; v < a.E / 8; v += stride) {
      float wv[8], uv[8];
      load8(w + 8 * v, wv);
      load8(u + 8 * v, uv);
#pragma unroll
      for (int j = 0; j < 8; ++j) wv[j] = __fmul_rn(wv[j], a.decay);
      round8<T>(wv);
      round8<T>(uv);
#pragma unroll
      for (int j = 0; j < 8; ++j) wv[j] = __fmaf_rn(a.alpha, uv[j], wv[j]);
      round8<T>(wv);
      store8(w + 8 * v, wv);
    }
  } else {
    for (long long e = first; e < a.E; e += stride) {
      const float w1 = round_to<T>(__fmul_rn(to_f32(w[e]), a.decay));
      const float uv = round_to<T>(to_f32(u[e]));
      w[e] = from_f32<T>(__fmaf_rn(a.alpha, uv, w1));
    }
  }
}

}  // namespace ps
