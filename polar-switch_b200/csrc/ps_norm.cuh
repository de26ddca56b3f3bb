// HBM-bound helper kernels of the circuit:
//   * Frobenius normalisation  Xh = fp16( fp32(X) / (||fp32(X)||_F + eps) )
//     (polar_switch/__init__.py:34-35), two passes: per-chunk sums of squares
//     into a caller-provided scratch array, then a scale + cast pass that also
//     zero-fills any alignment padding;
//   * copy-out of a padded FP16 result into the caller's dtype and shape
//     (polar_switch/__init__.py:168, `.to(X.dtype).reshape(X.shape)`);
//   * Q = Z + a*I for Gram Newton-Schulz (polar_switch/gram_newton_schulz.py:107),
//     with torch's FP16 semantics: fp16(Z_ii + fp16(a)).
#pragma once

#include "ps_ptx.cuh"

namespace ps {

enum DType : int { kF16 = 0, kF32 = 1, kBF16 = 2, kF64 = 3 };

constexpr int NORM_THREADS = 256;

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_f32<float>(float v) {
  return v;
}
template <>
__device__ __forceinline__ float to_f32<double>(double v) {
  return static_cast<float>(v);  // X.float() first, as the reference does
}

template <typename T>
__device__ __forceinline__ T from_f16(__half h);
template <>
__device__ __forceinline__ __half from_f16<__half>(__half h) {
  return h;
}
template <>
__device__ __forceinline__ __nv_bfloat16 from_f16<__nv_bfloat16>(__half h) {
  return __float2bfloat16_rn(__half2float(h));
}
template <>
__device__ __forceinline__ float from_f16<float>(__half h) {
  return __half2float(h);
}
template <>
__device__ __forceinline__ double from_f16<double>(__half h) {
  return static_cast<double>(__half2float(h));
}

// Deterministic block sum (fixed shuffle tree, warps combined in order).
__device__ __forceinline__ double block_sum(double v, double* s_warp) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) s_warp[warp] = v;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x == 0) {
    for (int w = 0; w < (blockDim.x >> 5); ++w) t += s_warp[w];
  }
  return t;
}

// 16-byte vector of T unpacked to floats (VW = 16 / sizeof(T) values).
template <typename T>
struct Vec16 {
  static constexpr int VW = 16 / sizeof(T);
  __device__ __forceinline__ static void load(const T* p, float (&f)[VW]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const T* t = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < VW; ++i) f[i] = to_f32(t[i]);
  }
};

__device__ __forceinline__ bool is_aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Pass 1: partial[l * chunks + chunk] = sum of squares of one chunk of matrix l.
// `flat` means the matrix is one contiguous run of R*C elements.
template <typename T>
__global__ void __launch_bounds__(NORM_THREADS)
    ps_norm_partial_kernel(const T* __restrict__ x, long long R, long long C, long long sL,
                           long long sR, long long sC, int flat, int chunks,
                           double* __restrict__ partial) {
  __shared__ double s_warp[NORM_THREADS / 32];
  const int l = blockIdx.y, chunk = blockIdx.x;
  const T* xm = x + static_cast<long long>(l) * sL;
  double acc = 0.0;
  if (flat) {
    constexpr int VW = Vec16<T>::VW;
    const long long E = R * C;
    // chunk boundaries on whole 16-byte vectors
    long long per = (E + chunks - 1) / chunks;
    per = (per + VW - 1) / VW * VW;
    const long long beg = chunk * per;
    const long long end = beg + per < E ? beg + per : E;
    if (is_aligned16(xm) && beg < end) {
      // FP32 partial sums per thread (a few hundred terms), FP64 across threads.
      float a0 = 0.f, a1 = 0.f;
      const long long nvec = (end - beg) / VW;
      const T* base = xm + beg;
      long long v = threadIdx.x;
      for (; v + NORM_THREADS < nvec; v += 2 * NORM_THREADS) {
        float f0[VW], f1[VW];
        Vec16<T>::load(base + v * VW, f0);
        Vec16<T>::load(base + (v + NORM_THREADS) * VW, f1);
#pragma unroll
        for (int i = 0; i < VW; ++i) {
          a0 = fmaf(f0[i], f0[i], a0);
          a1 = fmaf(f1[i], f1[i], a1);
        }
      }
      for (; v < nvec; v += NORM_THREADS) {
        float f0[VW];
        Vec16<T>::load(base + v * VW, f0);
#pragma unroll
        for (int i = 0; i < VW; ++i) a0 = fmaf(f0[i], f0[i], a0);
      }
      for (long long e = beg + nvec * VW + threadIdx.x; e < end; e += NORM_THREADS) {
        const float f = to_f32(xm[e]);
        a1 = fmaf(f, f, a1);
      }
      acc = static_cast<double>(a0) + static_cast<double>(a1);
    } else {
      for (long long e = beg + threadIdx.x; e < end; e += NORM_THREADS) {
        const float v = to_f32(xm[e]);
        acc += static_cast<double>(v) * v;
      }
    }
  } else {
    const long long per = (R + chunks - 1) / chunks;
    const long long rbeg = chunk * per;
    const long long rend = rbeg + per < R ? rbeg + per : R;
    for (long long r = rbeg; r < rend; ++r) {
      for (long long c = threadIdx.x; c < C; c += NORM_THREADS) {
        const float v = to_f32(xm[r * sR + c * sC]);
        acc += static_cast<double>(v) * v;
      }
    }
  }
  const double tot = block_sum(acc, s_warp);
  if (threadIdx.x == 0) partial[static_cast<long long>(l) * chunks + chunk] = tot;
}

// Pass 2: Xh[l] (Rp x Cp, FP16, zero padding) = X[l] / (norm_l + eps).
template <typename T>
__global__ void __launch_bounds__(NORM_THREADS)
    ps_scale_cast_kernel(const T* __restrict__ x, long long R, long long C, long long sL,
                         long long sR, long long sC, int flat, const double* __restrict__ partial,
                         int chunks, float eps, __half* __restrict__ xh, long long Rp,
                         long long Cp) {
  __shared__ float s_den;
  const int l = blockIdx.y;
  if (threadIdx.x < 32) {
    double s = 0.0;
    for (int i = threadIdx.x; i < chunks; i += 32) s += partial[static_cast<long long>(l) * chunks + i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) {
      const float nrm = static_cast<float>(sqrt(s));
      s_den = nrm + eps;  // FP32 add, as X.norm(...) + epsilon
    }
  }
  __syncthreads();
  const float den = s_den;
  const T* xm = x + static_cast<long long>(l) * sL;
  __half* out = xh + static_cast<long long>(l) * Rp * Cp;
  if (flat && Rp == R && Cp == C) {
    constexpr int VW = Vec16<T>::VW;
    const long long E = R * C;
    const long long stride = static_cast<long long>(gridDim.x) * NORM_THREADS;
    long long tail = 0;
    if (is_aligned16(xm) && is_aligned16(out)) {
      const long long nvec = E / VW;
      for (long long v = static_cast<long long>(blockIdx.x) * NORM_THREADS + threadIdx.x; v < nvec;
           v += stride) {
        float f[VW];
        Vec16<T>::load(xm + v * VW, f);
        uint32_t h[VW / 2];
#pragma unroll
        for (int i = 0; i < VW / 2; ++i)
          h[i] = pack_half2(__fdiv_rn(f[2 * i], den), __fdiv_rn(f[2 * i + 1], den));
        if constexpr (VW == 8) {
          *reinterpret_cast<uint4*>(out + v * VW) = make_uint4(h[0], h[1], h[2], h[3]);
        } else if constexpr (VW == 4) {
          *reinterpret_cast<uint2*>(out + v * VW) = make_uint2(h[0], h[1]);
        } else {
          *reinterpret_cast<uint32_t*>(out + v * VW) = h[0];
        }
      }
      tail = nvec * VW;
    }
    for (long long e = tail + static_cast<long long>(blockIdx.x) * NORM_THREADS + threadIdx.x; e < E;
         e += stride)
      out[e] = __float2half_rn(__fdiv_rn(to_f32(xm[e]), den));
  } else {
    const long long E = Rp * Cp;
    for (long long e = static_cast<long long>(blockIdx.x) * NORM_THREADS + threadIdx.x; e < E;
         e += static_cast<long long>(gridDim.x) * NORM_THREADS) {
      const long long r = e / Cp, c = e - r * Cp;
      float v = 0.f;
      if (r < R && c < C) v = __fdiv_rn(to_f32(xm[r * sR + c * sC]), den);
      out[e] = __float2half_rn(v);
    }
  }
}

// y[l] (R x C, contiguous, type T) = xh[l][:R, :C] (FP16, Rp x Cp).
template <typename T>
__global__ void __launch_bounds__(NORM_THREADS)
    ps_copy_out_kernel(const __half* __restrict__ xh, long long Rp, long long Cp, long long R,
                       long long C, long long L, T* __restrict__ y) {
  const long long E = L * R * C;
  for (long long e = static_cast<long long>(blockIdx.x) * NORM_THREADS + threadIdx.x; e < E;
       e += static_cast<long long>(gridDim.x) * NORM_THREADS) {
    const long long l = e / (R * C);
    const long long rc = e - l * R * C;
    const long long r = rc / C, c = rc - r * C;
    y[e] = from_f16<T>(xh[l * Rp * Cp + r * Cp + c]);
  }
}

// out = in + fp16(a) * I, FP16, elementwise (torch semantics of `Z + a * I`).
__global__ void __launch_bounds__(NORM_THREADS)
    ps_add_diag_kernel(const __half* __restrict__ in, __half* __restrict__ out, long long L,
                       long long n, float a) {
  const long long E = L * n * n;
  const float ah = __half2float(__float2half_rn(a));
  for (long long e = static_cast<long long>(blockIdx.x) * NORM_THREADS + threadIdx.x; e < E;
       e += static_cast<long long>(gridDim.x) * NORM_THREADS) {
    const long long rc = e % (n * n);
    const long long r = rc / n, c = rc - r * n;
    const __half v = in[e];
    out[e] = (r == c) ? __float2half_rn(__half2float(v) + ah) : v;
  }
}

// Self-test of the bounded-wait path: waits on an mbarrier that nothing
// arrives at; must give up after `limit` cycles and record the status code.
__global__ void ps_selftest_wait_kernel(int* status, long long limit) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_wait_bounded(&bar, 0, &abort_flag, status, kStatusSelftestTimeout, limit);
  }
  __syncthreads();
}

}  // namespace ps
