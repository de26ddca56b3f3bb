// HBM-bound helper kernels of the circuit:
//   * Frobenius normalisation  Xh = fp16( fp32(X) / (||fp32(X)||_F + eps) )
//     (polar_switch/__init__.py:34-35), two passes: per-chunk sums of squares
//     into a caller-provided scratch array (contiguous input over fixed
//     chunks, so a matrix normalises to the same bits in any batch), then a
//     scale + cast pass that also zero-fills any alignment padding;
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

// ---------------------------------------------------------------- canonical reduction
// The sum of squares of a contiguous matrix of E elements is reduced over
// fixed chunks of norm_chunk_elems(E) elements, a function of E alone, so the
// result does not depend on the batch around the matrix: per chunk, each
// thread accumulates in FP32 the 16-byte vectors tid, tid + NORM_THREADS, ...
// (a few dozen terms), then a fixed FP64 tree over the block; per matrix, lane
// i of one warp sums chunks i, i + 32, ... in FP64, then a fixed shuffle tree.
constexpr int NORM_CHUNK = 12288;       // elements per chunk (48 KB of FP32)
constexpr int NORM_MAX_CHUNKS = 1024;   // chunks per matrix at most

__host__ __device__ inline long long norm_chunk_elems(long long E) {
  const long long nch = (E + NORM_CHUNK - 1) / NORM_CHUNK;
  long long mult = (nch + NORM_MAX_CHUNKS - 1) / NORM_MAX_CHUNKS;
  if (mult < 1) mult = 1;
  return NORM_CHUNK * mult;
}

// Sum of squares of n contiguous elements (valid in thread 0). 16-byte vector
// loads, eight in flight per thread, need an aligned start; an unaligned run
// is read element by element in the same order, so the sum is the same.
template <typename T>
__device__ __forceinline__ double chunk_sumsq(const T* p, long long n, double* s_warp) {
  constexpr int VW = Vec16<T>::VW;
  float a = 0.f;
  const long long nvec = n / VW;
  if (is_aligned16(p)) {
    long long v = threadIdx.x;
    for (; v + 7 * NORM_THREADS < nvec; v += 8 * NORM_THREADS) {
      float f[8][VW];
#pragma unroll
      for (int k = 0; k < 8; ++k) Vec16<T>::load(p + (v + k * NORM_THREADS) * VW, f[k]);
#pragma unroll
      for (int k = 0; k < 8; ++k)
#pragma unroll
        for (int i = 0; i < VW; ++i) a = fmaf(f[k][i], f[k][i], a);
    }
    for (; v < nvec; v += NORM_THREADS) {
      float f[VW];
      Vec16<T>::load(p + v * VW, f);
#pragma unroll
      for (int i = 0; i < VW; ++i) a = fmaf(f[i], f[i], a);
    }
  } else {
    for (long long v = threadIdx.x; v < nvec; v += NORM_THREADS) {
#pragma unroll
      for (int i = 0; i < VW; ++i) {
        const float f = to_f32(p[v * VW + i]);
        a = fmaf(f, f, a);
      }
    }
  }
  for (long long e = nvec * VW + threadIdx.x; e < n; e += NORM_THREADS) {
    const float f = to_f32(p[e]);
    a = fmaf(f, f, a);
  }
  return block_sum(static_cast<double>(a), s_warp);
}

// Sum of one matrix's `nch` chunk sums in a fixed order (lane i adds chunks
// i, i + 32, ..., then a fixed shuffle tree); called by one full warp, valid in
// every lane. Loads run ahead of the (ordered) additions.
__device__ __forceinline__ double ordered_sum(const double* partial_m, int nch) {
  const int lane = threadIdx.x & 31;
  double s = 0.0;
  int i = lane;
  for (; i + 32 * 7 < nch; i += 32 * 8) {
    double v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = partial_m[i + 32 * k];
#pragma unroll
    for (int k = 0; k < 8; ++k) s += v[k];
  }
  for (; i < nch; i += 32) s += partial_m[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

// Denominator ||X||_F + eps of one matrix from its chunk sums (one full warp).
__device__ __forceinline__ float norm_den(const double* partial_m, int nch, float eps) {
  const float nrm = static_cast<float>(sqrt(ordered_sum(partial_m, nch)));
  return nrm + eps;  // FP32 add, as X.norm(...) + epsilon
}

// sums[l] = ordered_sum of matrix l's chunk sums (one warp per matrix).
__global__ void ps_sum_partials_kernel(const double* __restrict__ partial, int chunks, long long L,
                                       double* __restrict__ sums) {
  const long long l = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (l >= L) return;
  const double s = ordered_sum(partial + l * chunks, chunks);
  if ((threadIdx.x & 31) == 0) sums[l] = s;
}

// Pass 1: partial[l * chunks + chunk] = sum of squares of one chunk of matrix l.
// Contiguous matrices (`flat`) use the canonical chunks of `chunk_elems`
// elements; strided ones are split into `chunks` row ranges.
template <typename T>
__device__ __forceinline__ void norm_partial_body(const T* __restrict__ x, long long R, long long C,
                                                  long long sL, long long sR, long long sC, int flat,
                                                  int chunks, long long chunk_elems,
                                                  double* __restrict__ partial, long long l,
                                                  long long chunk) {
  __shared__ double s_warp[NORM_THREADS / 32];
  const T* xm = x + l * sL;
  double tot;
  if (flat) {
    const long long E = R * C;
    const long long beg = chunk * chunk_elems;
    const long long n = beg < E ? (E - beg < chunk_elems ? E - beg : chunk_elems) : 0;
    tot = chunk_sumsq(xm + beg, n, s_warp);
  } else {
    double acc = 0.0;
    const long long per = (R + chunks - 1) / chunks;
    const long long rbeg = chunk * per;
    const long long rend = rbeg + per < R ? rbeg + per : R;
    for (long long r = rbeg; r < rend; ++r) {
      for (long long c = threadIdx.x; c < C; c += NORM_THREADS) {
        const float v = to_f32(xm[r * sR + c * sC]);
        acc += static_cast<double>(v) * v;
      }
    }
    tot = block_sum(acc, s_warp);
  }
  if (threadIdx.x == 0) partial[l * chunks + chunk] = tot;
}

template <typename T>
__global__ void __launch_bounds__(NORM_THREADS)
    ps_norm_partial_kernel(const T* __restrict__ x, long long R, long long C, long long sL,
                           long long sR, long long sC, int flat, int chunks, long long chunk_elems,
                           double* __restrict__ partial) {
  norm_partial_body(x, R, C, sL, sR, sC, flat, chunks, chunk_elems, partial, blockIdx.y, blockIdx.x);
}

// 8 consecutive elements of T (16-byte aligned) as floats.
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&f)[8]) {
  constexpr int VW = Vec16<T>::VW;
  if constexpr (VW >= 8) {
    Vec16<T>::load(p, f);
  } else {
#pragma unroll
    for (int k = 0; k < 8 / VW; ++k) {
      float g[VW];
      Vec16<T>::load(p + k * VW, g);
#pragma unroll
      for (int i = 0; i < VW; ++i) f[k * VW + i] = g[i];
    }
  }
}

__device__ __forceinline__ uint4 scale8(const float (&f)[8], float den) {
  return make_uint4(pack_half2(__fdiv_rn(f[0], den), __fdiv_rn(f[1], den)),
                    pack_half2(__fdiv_rn(f[2], den), __fdiv_rn(f[3], den)),
                    pack_half2(__fdiv_rn(f[4], den), __fdiv_rn(f[5], den)),
                    pack_half2(__fdiv_rn(f[6], den), __fdiv_rn(f[7], den)));
}

// Pass 2: Xh[l] (Rp x Cp, FP16, zero padding) = X[l] / (norm_l + eps).
template <typename T>
__device__ __forceinline__ void scale_cast_body(const T* __restrict__ x, long long R, long long C,
                                                long long sL, long long sR, long long sC, int flat,
                                                const double* __restrict__ partial, int chunks,
                                                float eps, __half* __restrict__ xh, long long Rp,
                                                long long Cp, long long l, long long bx,
                                                long long gx) {
  __shared__ float s_den;
  if (threadIdx.x < 32) {
    // No partial sums: a plain FP16 rounding (denominator 1).
    const float den = partial ? norm_den(partial + l * chunks, chunks, eps)
                              : 1.0f;
    if (threadIdx.x == 0) s_den = den;
  }
  __syncthreads();
  const float den = s_den;
  const T* xm = x + l * sL;
  __half* out = xh + l * Rp * Cp;
  if (flat && Rp == R && Cp == C) {
    const long long E = R * C;
    const long long stride = gx * NORM_THREADS;
    long long tail = 0;
    if (is_aligned16(xm) && is_aligned16(out)) {
      // 8 elements per 16-byte store, two groups in flight per thread.
      const long long n8 = E / 8;
      long long v = bx * NORM_THREADS + threadIdx.x;
      for (; v + stride < n8; v += 2 * stride) {
        float f0[8], f1[8];
        load8(xm + v * 8, f0);
        load8(xm + (v + stride) * 8, f1);
        *reinterpret_cast<uint4*>(out + v * 8) = scale8(f0, den);
        *reinterpret_cast<uint4*>(out + (v + stride) * 8) = scale8(f1, den);
      }
      for (; v < n8; v += stride) {
        float f[8];
        load8(xm + v * 8, f);
        *reinterpret_cast<uint4*>(out + v * 8) = scale8(f, den);
      }
      tail = n8 * 8;
    }
    for (long long e = tail + bx * NORM_THREADS + threadIdx.x; e < E;
         e += stride)
      out[e] = __float2half_rn(__fdiv_rn(to_f32(xm[e]), den));
  } else {
    const long long E = Rp * Cp;
    for (long long e = bx * NORM_THREADS + threadIdx.x; e < E;
         e += gx * NORM_THREADS) {
      const long long r = e / Cp, c = e - r * Cp;
      float v = 0.f;
      if (r < R && c < C) v = __fdiv_rn(to_f32(xm[r * sR + c * sC]), den);
      out[e] = __float2half_rn(v);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(NORM_THREADS)
    ps_scale_cast_kernel(const T* __restrict__ x, long long R, long long C, long long sL,
                         long long sR, long long sC, int flat, const double* __restrict__ partial,
                         int chunks, float eps, __half* __restrict__ xh, long long Rp,
                         long long Cp) {
  scale_cast_body(x, R, C, sL, sR, sC, flat, partial, chunks, eps, xh, Rp, Cp, blockIdx.y, blockIdx.x,
                  gridDim.x);
}

// Both passes over up to NORM_BATCH_MAX problems of one input type, one launch
// per pass (the normalisations that open a grouped circuit). The 1-D grid is
// the concatenation of the problems' own grids, problem i owning blocks
// [b0, b0 + L * per) with `per` blocks per matrix: its chunks in pass 1, its
// scale-and-cast blocks in pass 2. Each matrix sees exactly the chunking and
// arithmetic of the single-problem kernels, so the results are bit-identical.
constexpr int NORM_BATCH_MAX = 8;

struct NormBatchProblem {
  const void* x;
  __half* xh;
  double* partial;
  long long R, C, sL, sR, sC, Rp, Cp, chunk_elems;
  long long b0;   // first block of this problem in the launch
  long long per;  // blocks per matrix
  int flat, chunks;
};

struct NormBatch {
  NormBatchProblem p[NORM_BATCH_MAX];
  int count;
  float eps;
};

__device__ __forceinline__ int norm_batch_problem(const NormBatch& b, long long blk) {
  int pi = 0;
  while (pi + 1 < b.count && blk >= b.p[pi + 1].b0) ++pi;
  return pi;
}

template <typename T>
__global__ void __launch_bounds__(NORM_THREADS)
    ps_norm_partial_batched_kernel(const __grid_constant__ NormBatch b) {
  const long long blk = blockIdx.x;
  const NormBatchProblem& q = b.p[norm_batch_problem(b, blk)];
  const long long local = blk - q.b0;
  norm_partial_body(static_cast<const T*>(q.x), q.R, q.C, q.sL, q.sR, q.sC, q.flat, q.chunks,
                    q.chunk_elems, q.partial, local / q.per, local % q.per);
}

template <typename T>
__global__ void __launch_bounds__(NORM_THREADS)
    ps_scale_cast_batched_kernel(const __grid_constant__ NormBatch b) {
  const long long blk = blockIdx.x;
  const NormBatchProblem& q = b.p[norm_batch_problem(b, blk)];
  const long long local = blk - q.b0;
  scale_cast_body(static_cast<const T*>(q.x), q.R, q.C, q.sL, q.sR, q.sC, q.flat, q.partial, q.chunks,
                  b.eps, q.xh, q.Rp, q.Cp, local / q.per, local % q.per, q.per);
}

// Both passes of the normalisation with one read of the input ("fused"), for
// contiguous matrices without padding. A persistent grid walks the chunks of
// all problems in order; a CTA loads its chunk into shared memory while
// summing its squares exactly as ps_norm_partial_kernel does (same vectors per
// thread, same FP32 order, same FP64 block tree), publishes the sum and bumps
// its matrix's counter, waits (bounded) until every chunk of that matrix is
// summed, forms the denominator as ps_scale_cast_kernel does (norm_den) and
// writes its chunk's FP16 values from shared memory. So the bits are those of
// the two-pass kernels, and the input crosses HBM once (6 instead of 10 bytes
// per FP32 element).
//
// A CTA waits only for chunks of its own matrix, which sit at most
// `chunks - 1` places after its own in the order; with every chunk count at
// most the grid size and all CTAs resident, the earliest unfinished matrix
// always has all its chunks held by running CTAs, so the waits end.
struct NormFusedProblem {
  const void* x;        // (L, E) contiguous input
  __half* xh;           // (L, E) FP16 output
  double* partial;      // L * chunks chunk sums
  unsigned* count;      // L counters, zero on entry
  long long E;          // elements per matrix
  long long t0;         // first chunk of this problem in the launch
  int chunks;           // chunks per matrix (chunk size NORM_CHUNK)
};

struct NormFused {
  NormFusedProblem p[NORM_BATCH_MAX];
  int count;
  long long total;      // chunks of all problems
  float eps;
  int* status;
  long long wait_limit;
};

template <typename T>
__global__ void __launch_bounds__(NORM_THREADS)
    ps_normalize_fused_kernel(const __grid_constant__ NormFused F) {
  extern __shared__ uint4 s_chunk[];  // NORM_CHUNK elements of T
  __shared__ double s_warp[NORM_THREADS / 32];
  __shared__ float s_den;
  __shared__ int s_ok;
  constexpr int VW = Vec16<T>::VW;
  T* sdata = reinterpret_cast<T*>(s_chunk);
  for (long long t = blockIdx.x; t < F.total; t += gridDim.x) {
    int pi = 0;
    while (pi + 1 < F.count && t >= F.p[pi + 1].t0) ++pi;
    const NormFusedProblem& q = F.p[pi];
    const long long local = t - q.t0;
    const long long l = local / q.chunks, c = local - l * q.chunks;
    const long long beg = c * NORM_CHUNK;
    const long long n = q.E - beg < NORM_CHUNK ? q.E - beg : NORM_CHUNK;
    const T* src = static_cast<const T*>(q.x) + l * q.E + beg;
    // Sum of squares in chunk_sumsq's order, keeping the chunk in shared memory.
    float a = 0.f;
    const long long nvec = n / VW;
    long long v = threadIdx.x;
    for (; v + 7 * NORM_THREADS < nvec; v += 8 * NORM_THREADS) {
      uint4 u[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) u[k] = __ldg(reinterpret_cast<const uint4*>(src) + v + k * NORM_THREADS);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        s_chunk[v + k * NORM_THREADS] = u[k];
        const T* e = reinterpret_cast<const T*>(&u[k]);
#pragma unroll
        for (int i = 0; i < VW; ++i) {
          const float f = to_f32(e[i]);
          a = fmaf(f, f, a);
        }
      }
    }
    for (; v < nvec; v += NORM_THREADS) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(src) + v);
      s_chunk[v] = u;
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int i = 0; i < VW; ++i) {
        const float f = to_f32(e[i]);
        a = fmaf(f, f, a);
      }
    }
    for (long long e = nvec * VW + threadIdx.x; e < n; e += NORM_THREADS) {
      const T xv = src[e];
      sdata[e] = xv;
      const float f = to_f32(xv);
      a = fmaf(f, f, a);
    }
    const double tot = block_sum(static_cast<double>(a), s_warp);
    if (threadIdx.x == 0) {
      q.partial[l * q.chunks + c] = tot;
      __threadfence();
      atomicAdd(q.count + l, 1u);
      const unsigned need = static_cast<unsigned>(q.chunks);
      int ok = 1;
      if (ld_acquire_gpu_u32(q.count + l) < need) {
        const long long start = clock64();
        while (ld_acquire_gpu_u32(q.count + l) < need) {
          __nanosleep(64);
          if (*reinterpret_cast<volatile int*>(F.status) != 0 || clock64() - start > F.wait_limit) {
            atomicCAS(F.status, 0, kStatusNormalizeTimeout);
            ok = 0;
            break;
          }
        }
      }
      s_ok = ok;
    }
    __syncthreads();
    if (!s_ok) return;
    if (threadIdx.x < 32) {
      const float den = norm_den(q.partial + l * q.chunks, q.chunks, F.eps);
      if (threadIdx.x == 0) s_den = den;
    }
    __syncthreads();
    const float den = s_den;
    __half* out = q.xh + l * q.E + beg;
    const long long n8 = n / 8;
    for (long long g = threadIdx.x; g < n8; g += NORM_THREADS) {
      float f[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] = to_f32(sdata[g * 8 + i]);
      *reinterpret_cast<uint4*>(out + g * 8) = scale8(f, den);
    }
    for (long long e = n8 * 8 + threadIdx.x; e < n; e += NORM_THREADS)
      out[e] = __float2half_rn(__fdiv_rn(to_f32(sdata[e]), den));
    __syncthreads();  // the next chunk overwrites s_chunk
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
