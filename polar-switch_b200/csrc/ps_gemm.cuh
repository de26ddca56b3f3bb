// One persistent, warp-specialised tcgen05 GEMM family that implements every
// dense contraction of a Polar Switch circuit:
//
//   symmetric  D = alpha * A . B^T + beta * C + diag * I     (gram, square,
//              only tiles on or above the block diagonal are computed; the
//              epilogue writes each off-diagonal 128x128 block twice, once
//              transposed, unless the result is kept as upper-triangle blocks)
//   general    D = A . B^T + beta * C                          (apply)
//
// "B^T" is in the UMMA sense (B supplies N rows of K): a K-major B tile is
// read from the rows of a row-major matrix (A . A^T for a squared buffer, the
// Gram X . X^T), an MN-major B tile from its columns, which makes the product
// exactly A @ B (products of two different matrices, apply).
//
// Operands are FP16 in HBM, staged by TMA into 128-byte-swizzled shared
// memory, multiplied by tcgen05.mma (kind::f16) into FP32 accumulators in
// TMEM, and the epilogue does alpha/beta*C/diag in FP32 followed by exactly
// one rounding to FP16 (optionally widened to FP32/BF16 for the final output).
//
// Roles (320 threads, one CTA per SM, persistent over a static tile list that
// may span several problems, see GemmBatch):
//   warp 0 lane 0   TMA producer, STAGES-deep smem ring
//   warp 1          TMEM allocator; lane 0 issues the UMMAs
//   warps 2..9      epilogue, two warps per TMEM lane quarter, 128 columns
//                   each: tcgen05.ld -> FP32 math -> swizzled smem -> TMA
//                   store (plus the mirrored store for symmetric tiles)
//
// Reference behaviour this follows: polar_switch/triton_kernels.py:24-57 (one
// owner per symmetric tile, FP32 epilogue alpha*acc + beta*C then + diag,
// single FP16 store and a transposed mirror store) and
// polar_switch/gemm_symmetric_fused.py:45-76 (mirror only off the diagonal,
// diagonal shift only where the tile meets the diagonal).
#pragma once

#include "ps_ptx.cuh"

namespace ps {

constexpr int BM = 128;           // UMMA M (TMEM lanes)
constexpr int BN = 256;           // UMMA N (TMEM columns per accumulator)
constexpr int BK = 64;            // 64 halves = one 128-byte swizzle row
constexpr int STAGES = 4;
constexpr int UMMA_K = 16;
constexpr int A_STAGE_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_STAGE_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int MN_ATOM_BYTES = 64 * BK * 2;  // one 64(MN) x 64(K) MN-major box: 8 KB
constexpr int NUM_EPI_WARPS = 8;   // two per TMEM lane quarter, 128 columns each
constexpr int NUM_THREADS = 64 + 32 * NUM_EPI_WARPS;
constexpr int EPI_WARP_BYTES = 4096;
constexpr int SMEM_OPERANDS = STAGES * STAGE_BYTES;
constexpr int SMEM_EPI = NUM_EPI_WARPS * EPI_WARP_BYTES;
constexpr int SMEM_CTRL = 256;
constexpr int SMEM_TOTAL = SMEM_OPERANDS + SMEM_EPI + SMEM_CTRL + 1024;  // +1 KB alignment slack
constexpr uint32_t TMEM_COLS = 2 * BN;   // double-buffered accumulator
constexpr long long kDefaultWaitLimit = 1ll << 32;  // ~2 s of SM clock

enum OutType : int { kOutF16 = 0, kOutF32 = 1, kOutBF16 = 2 };

struct GemmArgs {
  int M, N, K, L;            // D is M x N per matrix, L matrices
  int tiles_m, tiles_n;      // general mode: tile grid
  int tb;                    // symmetric mode: number of 128-row blocks
  int tiles_per_mat, total_tiles;
  int group_m;               // general mode: M-tiles per rasterisation group
  float alpha, beta, diag;
  const __half* C;           // addend (FP16), may alias D in symmetric mode
  long long c_ld, c_bs;      // addend leading dimension / batch stride (elements)
  int has_addend, has_diag;
  // Triangle storage: a_tri / b_tri mark operands held as upper-triangle
  // blocks (read through the second maps, see tri_transposed); store_mirror = 0
  // keeps a symmetric result that way (no transposed stores).
  int a_tri, b_tri, store_mirror;
  // Symmetric A . A^T with both operands read through identical maps: the
  // CTA-pair kernel then stages a diagonal pair tile's rows once.
  int same_ab;
  // CTA-pair path only: the operand map is a 4-D chunked map (one TMA per
  // 128-wide K stage, see ps_gemm2.cuh); the one-CTA kernel ignores these.
  int a_chunk, b_chunk, a2_chunk, b2_chunk;
  // CTA-pair path only: Muon update of a parameter bank in place of the
  // output store (see pair::PairArgs).
  int upd, p_dtype;
  void* P;
  long long p_ld, p_bs;
  float decay, upd_alpha;
  int* status;               // device status word
  long long wait_limit;      // cycles before a bounded wait gives up
};

// Symmetric tiles: row block bi owns the tiles starting at block columns
// j = bi, bi + 2, ... < tb (each tile covers blocks j and j + 1). Above
// SYM_BAND row blocks they are visited in bands of SYM_BAND row blocks; inside
// a band by start column j, and for each j by row. CTAs that run at the same time then share a few A row
// panels and B column panels, so a long K streams each panel from DRAM about
// once per band instead of once per tile.
#ifndef PS_SYM_BAND
#define PS_SYM_BAND 16
#endif
constexpr int SYM_BAND = PS_SYM_BAND;

// Rows x in [lo, hi) with x % 2 == par.
__device__ __forceinline__ int count_parity(int lo, int hi, int par) {
  return ((hi - par + 1) >> 1) - ((lo - par + 1) >> 1);
}

__device__ __forceinline__ void decode_sym(int tb, int r, int& bi, int& j) {
  int lo = 0, hi = 0;
  while (true) {
    hi = min(lo + SYM_BAND, tb);
    int total = 0;
    for (int x = lo; x < hi; ++x) total += (tb - x + 1) >> 1;
    if (r < total) break;
    r -= total;
    lo = hi;
  }
  // Start columns inside the band: the count of rows grows with j ...
  for (j = lo; j < tb; ++j) {
    const int par = j & 1;
    const int cnt = count_parity(lo, min(hi, j + 1), par);
    if (r < cnt) {
      bi = lo + ((lo & 1) != par) + 2 * r;
      return;
    }
    r -= cnt;
    if (j >= hi - 1) break;
  }
  // ... and from j = hi on alternates between the band's even and odd rows.
  ++j;
  const int ce = count_parity(lo, hi, 0), co = count_parity(lo, hi, 1);
  const int k = r / (ce + co);
  j += 2 * k;
  r -= k * (ce + co);
  const int c_first = (j & 1) ? co : ce;
  if (r >= c_first) {
    r -= c_first;
    ++j;
  }
  bi = lo + ((lo & 1) != (j & 1)) + 2 * r;
}

// One launch covers up to MAX_BATCH problems of the same kernel variant (same
// operand majorness, symmetry and output type): their tiles are numbered one
// after the other (tile_start), and each tile reads its problem's maps and
// arguments. Circuits use this to run the Gram or apply of every bucket of a
// grouped call as one persistent launch.
#ifndef PS_MAX_BATCH
#define PS_MAX_BATCH 8
#endif
constexpr int MAX_BATCH = PS_MAX_BATCH;

struct alignas(64) GemmProblem {
  // tmA / tmB: boxes in the operand's native majorness (A_MN / B_MN);
  // tmA2 / tmB2: the other majorness, read only for triangle-stored operands.
  CUtensorMap tmA, tmA2, tmB, tmB2, tmD;
  GemmArgs args;
};

struct GemmBatch {
  GemmProblem p[MAX_BATCH];
  int tile_start[MAX_BATCH + 1];
  int count;
};

__device__ __forceinline__ int batch_problem(const GemmBatch& batch, int t) {
  int pi = 0;
  while (pi + 1 < batch.count && t >= batch.tile_start[pi + 1]) ++pi;
  return pi;
}

template <bool SYM>
__device__ __forceinline__ void decode_tile(const GemmArgs& a, int t, int& b, int& m0, int& n0) {
  b = t / a.tiles_per_mat;
  int r = t - b * a.tiles_per_mat;
  if (SYM) {
    int bi = 0, j;
    if (a.tb <= SYM_BAND) {
      // One band: plain row order, the cheapest decode (it sits on the UMMA
      // issuer's path between tiles, which matters when K is short).
      while (true) {
        const int cnt = (a.tb - bi + 1) >> 1;
        if (r < cnt) break;
        r -= cnt;
        ++bi;
      }
      j = bi + 2 * r;
    } else {
      decode_sym(a.tb, r, bi, j);
    }
    m0 = bi * BM;
    n0 = j * BM;
  } else {
    const int per_group = a.group_m * a.tiles_n;
    const int g = r / per_group;
    const int first = g * a.group_m;
    const int gsz = min(a.group_m, a.tiles_m - first);
    const int idx = r - g * per_group;
    m0 = (first + idx % gsz) * BM;
    n0 = (idx / gsz) * BN;
  }
}

// Triangle storage: a symmetric operand may be held as its 128x128 blocks on
// and above the diagonal only. For an operand tile whose 128-row blocks are
// lo..hi, k-block kb (a 128-wide block index) must then be read from the
// stored transposed block with the other majorness. K-native tiles hold rows
// of the operand (element (r, k) stored iff block(r) <= kb), MN-native tiles
// hold its columns. When a tile switches, a diagonal block it covers is read
// transposed too, which is exact: diagonal blocks are bit-symmetric (both
// triangles are computed by the same UMMA sums in the same order).
__device__ __forceinline__ bool tri_transposed(bool mn_native, int lo, int hi, int kb) {
  return mn_native ? (kb > lo) : (hi > kb);
}

template <int OUT>
struct OutTraits;
template <>
struct OutTraits<kOutF16> {
  static constexpr int kBytes = 2;
};
template <>
struct OutTraits<kOutBF16> {
  static constexpr int kBytes = 2;
};
template <>
struct OutTraits<kOutF32> {
  static constexpr int kBytes = 4;
};

// Convert 32 FP32 values of one output row to the output type, rounding to
// FP16 first (the circuit's single rounding) and widening afterwards.
template <int OUT>
__device__ __forceinline__ void convert_row(const float (&f)[32], uint32_t (&w)[32]) {
  if (OUT == kOutF16) {
#pragma unroll
    for (int j = 0; j < 16; ++j) w[j] = pack_half2(f[2 * j], f[2 * j + 1]);
  } else if (OUT == kOutBF16) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float lo = __half2float(__float2half_rn(f[2 * j]));
      const float hi = __half2float(__float2half_rn(f[2 * j + 1]));
      __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
      w[j] = *reinterpret_cast<uint32_t*>(&h);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) w[j] = __float_as_uint(__half2float(__float2half_rn(f[j])));
  }
}

// BATCHED = false: batch.count is 1 and the problem index is the constant 0, so
// the arguments are read at fixed parameter offsets (as cheap as plain kernel
// parameters); BATCHED = true looks the problem up per tile.
template <bool A_MN, bool B_MN, bool SYM, int OUT, bool BATCHED>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    ps_gemm_kernel(const __grid_constant__ GemmBatch batch) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzle atoms.
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* s_epi = smem + SMEM_OPERANDS;
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_epi + SMEM_EPI);
  uint64_t* full = bars;                  // [STAGES]
  uint64_t* empty = bars + STAGES;        // [STAGES]
  uint64_t* tfull = bars + 2 * STAGES;    // [2]
  uint64_t* tempty = tfull + 2;           // [2]
  uint64_t* drain = tempty + 2;           // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
#pragma unroll
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], NUM_EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    for (int pi = 0; pi < batch.count; ++pi) {
      const GemmProblem& P = batch.p[pi];
      tma_prefetch_desc(&P.tmA);
      tma_prefetch_desc(&P.tmB);
      tma_prefetch_desc(&P.tmD);
      if (P.args.a_tri) tma_prefetch_desc(&P.tmA2);
      if (P.args.b_tri) tma_prefetch_desc(&P.tmB2);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int total_tiles = batch.tile_start[batch.count];
  int* const status = batch.p[0].args.status;          // the same for every problem
  const long long wait_limit = batch.p[0].args.wait_limit;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        const int pi = BATCHED ? batch_problem(batch, t) : 0;
        const GemmProblem& P = batch.p[pi];
        const GemmArgs& args = P.args;
        const int num_kb = (args.K + BK - 1) / BK;
        int b, m0, n0;
        decode_tile<SYM>(args, t - batch.tile_start[pi], b, m0, n0);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, status,
                                 kStatusProducerTimeout, wait_limit)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = smem + stage * STAGE_BYTES;
          uint8_t* b_dst = a_dst + A_STAGE_BYTES;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          const int k0 = kb * BK;
          const int kb128 = k0 / BM;
          const bool at = args.a_tri && tri_transposed(A_MN, m0 / BM, m0 / BM, kb128);
          const bool bt = args.b_tri && tri_transposed(B_MN, n0 / BM, n0 / BM + 1, kb128);
          const CUtensorMap* ma = at ? &P.tmA2 : &P.tmA;
          const CUtensorMap* mb = bt ? &P.tmB2 : &P.tmB;
          if (A_MN == at) {  // K-major tile
            tma_load_3d(ma, a_dst, &full[stage], k0, m0, b);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_3d(ma, a_dst + j * MN_ATOM_BYTES, &full[stage], m0 + 64 * j, k0, b);
          }
          if (B_MN == bt) {
            tma_load_3d(mb, b_dst, &full[stage], k0, n0, b);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_3d(mb, b_dst + j * MN_ATOM_BYTES, &full[stage], n0 + 64 * j, k0, b);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let every load already in flight land before the CTA can exit.
        for (int s = 0; s < STAGES; ++s) {
          if (!(issued_mask & (1u << s))) continue;
          const uint32_t par = (issued_parity >> s) & 1u;
          const long long start = clock64();
          while (!mbar_try_wait(&full[s], par)) {
            if (clock64() - start > wait_limit) {
              if (status) atomicCAS(status, 0, kStatusDrainTimeout);
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued_any = false;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        const int pi = BATCHED ? batch_problem(batch, t) : 0;
        const GemmProblem& P = batch.p[pi];
        const GemmArgs& args = P.args;
        const int num_kb = (args.K + BK - 1) / BK;
        const int ncols_total = args.N;  // symmetric: N == M
        int b, m0, n0;
        decode_tile<SYM>(args, t - batch.tile_start[pi], b, m0, n0);
        int nvalid = ncols_total - n0;
        nvalid = nvalid > BN ? BN : nvalid;
        const int n_mma = (nvalid + 15) & ~15;
        if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1u, abort_flag, status,
                               kStatusMmaTimeout, wait_limit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, status, kStatusMmaTimeout,
                                 wait_limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_STAGE_BYTES;
          const int kb128 = (kb * BK) / BM;
          const bool a_mn = A_MN != (args.a_tri && tri_transposed(A_MN, m0 / BM, m0 / BM, kb128));
          const bool b_mn =
              B_MN != (args.b_tri && tri_transposed(B_MN, n0 / BM, n0 / BM + 1, kb128));
          const uint32_t idesc = make_idesc_f16(BM, n_mma, a_mn, b_mn);
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            const uint64_t ad = a_mn ? make_smem_desc_sw128(a_addr + kk * (UMMA_K * 128),
                                                            MN_ATOM_BYTES, 1024)
                                     : make_smem_desc_sw128(a_addr + kk * (UMMA_K * 2), 16, 1024);
            const uint64_t bd = b_mn ? make_smem_desc_sw128(b_addr + kk * (UMMA_K * 128),
                                                            MN_ATOM_BYTES, 1024)
                                     : make_smem_desc_sw128(b_addr + kk * (UMMA_K * 2), 16, 1024);
            umma_f16(d_tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          issued_any = true;
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && issued_any) {
        // Wait for the UMMAs already issued before TMEM is released.
        umma_commit(drain);
        const long long start = clock64();
        while (!mbar_try_wait(drain, 0)) {
          if (clock64() - start > wait_limit) {
            if (status) atomicCAS(status, 0, kStatusDrainTimeout);
            break;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    constexpr int OB = OutTraits<OUT>::kBytes;
    constexpr int ROW_BYTES = 32 * OB;              // one staged row: 64 B or 128 B
    constexpr int BUF_BYTES = 32 * ROW_BYTES;       // one 32 x 32 sub-tile
    // A slot holds what one chunk stores: the sub-tile, plus its transpose for
    // symmetric products. Slots rotate; one bulk group per slot.
    constexpr int SLOT_BYTES = SYM ? 2 * BUF_BYTES : BUF_BYTES;
    constexpr int NSLOT = EPI_WARP_BYTES / SLOT_BYTES;
    static_assert(NSLOT >= 1, "epilogue staging needs a slot");
    static_assert(!SYM || OUT == kOutF16, "symmetric products are stored in FP16");
    const int q = warp & 3;         // TMEM lane quarter this warp may access
    const int h = (warp - 2) >> 2;  // which 128 of the tile's 256 columns it drains
    const uint32_t stg = smem_u32(s_epi + (warp - 2) * EPI_WARP_BYTES);
    int acc = 0;
    uint32_t acc_phase = 0;
    int slot = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
      const int pi = BATCHED ? batch_problem(batch, t) : 0;
      const GemmProblem& P = batch.p[pi];
      const GemmArgs& args = P.args;
      const int ncols_total = args.N;  // symmetric: N == M
      int b, m0, n0;
      decode_tile<SYM>(args, t - batch.tile_start[pi], b, m0, n0);
      const int c_first = 4 * h;  // this warp's chunks: c_first .. c_first + 3
      int nvalid = ncols_total - (n0 + 32 * c_first);
      nvalid = nvalid > BN / 2 ? BN / 2 : nvalid;
      const int nchunks = nvalid > 0 ? (nvalid + 31) >> 5 : 0;
      const int row0 = m0 + 32 * q;       // first row of this warp's 32-row slab
      const int grow = row0 + lane;       // this thread's output row
      const bool row_ok = grow < args.M;
      const bool load_c = args.has_addend && row_ok;
      const __half* crow =
          args.has_addend ? args.C + static_cast<long long>(b) * args.c_bs +
                                static_cast<long long>(grow) * args.c_ld
                          : nullptr;
      // Pull this thread's addend row into L2 while the UMMAs of the tile run.
      if (load_c && nchunks > 0) {
        const int cb = n0 + 32 * c_first;
        const int ce = min(cb + nvalid, ncols_total);
        for (int cc = cb; cc < ce; cc += 64) prefetch_l2(crow + cc);
        prefetch_l2(crow + ce - 1);
      }
      // Addend vectors of chunk c, loaded coalesced: vector k is row 8k + lane/4,
      // columns 8 * (lane & 3) .. +7 of the warp's 32 x 32 sub-tile; they are
      // transposed to one row per lane through the staging slot.
      auto load_addend = [&](int c, uint4 (&dst)[4]) {
#pragma unroll
        for (int k = 0; k < 4; ++k) dst[k] = make_uint4(0, 0, 0, 0);
        if (!args.has_addend) return;
        const int gc = n0 + 32 * c + 8 * (lane & 3);
        const __half* cbat = args.C + static_cast<long long>(b) * args.c_bs;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int gr = row0 + 8 * k + (lane >> 2);
          if (gr >= args.M || gc >= ncols_total) continue;
          const __half* src = cbat + static_cast<long long>(gr) * args.c_ld + gc;
          if (gc + 8 <= ncols_total) {
            dst[k] = ld_global_v4(src);
          } else {
            __half* hv = reinterpret_cast<__half*>(&dst[k]);
            for (int e = 0; e < 8; ++e) hv[e] = (gc + e < ncols_total) ? src[e] : __float2half(0.f);
          }
        }
      };
      // Math, conversion and staging of chunk c (32 columns of this warp's
      // 32 rows), then one bulk group with its TMA store(s).
      auto process = [&](int c, const uint32_t (&v)[32], const uint4 (&av)[4]) {
        const int gcol0 = n0 + 32 * c;
        if (lane == 0) bulk_wait_read<NSLOT - 1>();  // the slot's previous stores have read it
        __syncwarp();
        const uint32_t sb = stg + slot * SLOT_BYTES;
        uint4 cv[4];
        if (args.has_addend) {
          // 64-byte FP16 rows, same swizzle as the output staging below
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int r = 8 * k + (lane >> 2), j = lane & 3;
            st_shared_v4(sb + r * 64 + ((j ^ ((r >> 1) & 3)) << 4), av[k].x, av[k].y, av[k].z,
                         av[k].w);
          }
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 4; ++j) cv[j] = ld_shared_v4(sb + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4));
        }
        float f[32];
        if (args.has_addend) {
          const __half* hv = reinterpret_cast<const __half*>(cv);
#pragma unroll
          for (int j = 0; j < 32; ++j)
            f[j] = fmaf(args.beta, __half2float(hv[j]), args.alpha * __uint_as_float(v[j]));
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) f[j] = args.alpha * __uint_as_float(v[j]);
        }
        if (SYM && args.has_diag) {
          const int d = grow - gcol0;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j == d) f[j] += args.diag;
        }
        uint32_t w[32];
        convert_row<OUT>(f, w);
        const bool mirror = SYM && args.store_mirror && (gcol0 / BM) != (m0 / BM);
        // With 64-byte output rows each lane only overwrites the addend row it
        // read itself; 128-byte output rows span other lanes' addend rows.
        if (ROW_BYTES != 64 && args.has_addend) __syncwarp();
        if (ROW_BYTES == 64) {
          // 64-byte rows, TMA SWIZZLE_64B: 16 B chunk j -> j ^ ((row >> 1) & 3)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int p = j ^ ((lane >> 1) & 3);
            st_shared_v4(sb + lane * 64 + p * 16, w[4 * j], w[4 * j + 1], w[4 * j + 2],
                         w[4 * j + 3]);
          }
        } else {
          // 128-byte rows, TMA SWIZZLE_128B: chunk j -> j ^ (row & 7)
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int p = j ^ (lane & 7);
            st_shared_v4(sb + lane * 128 + p * 16, w[4 * j], w[4 * j + 1], w[4 * j + 2],
                         w[4 * j + 3]);
          }
        }
        if (mirror) {
          // Transposed sub-tile: row t = column of D, column = lane (row of D).
          // Lane pairs swap halves so each lane stores 4 bytes.
          const uint32_t st = sb + BUF_BYTES;
          const int odd = lane & 1;
          const int cbyte = (lane & ~1) * 2;
#pragma unroll
          for (int p = 0; p < 16; ++p) {
            const uint32_t mine = w[p];
            const uint32_t send = odd ? (mine & 0xFFFFu) : (mine >> 16);
            const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, 1);
            const uint32_t val = odd ? ((recv & 0xFFFFu) | (mine & 0xFFFF0000u))
                                     : ((mine & 0xFFFFu) | (recv << 16));
            const int trow = 2 * p + odd;
            const int ch = (cbyte >> 4) ^ ((trow >> 1) & 3);
            st_shared_u32(st + trow * 64 + ch * 16 + (cbyte & 15), val);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (row0 < args.M && gcol0 < ncols_total) {
            tma_store_3d(&P.tmD, sb, gcol0, row0, b);
            if (mirror) tma_store_3d(&P.tmD, sb + BUF_BYTES, row0, gcol0, b);
          }
          bulk_commit();
        }
        slot = (slot + 1 == NSLOT) ? 0 : slot + 1;
      };
      // The accumulator may be reused as soon as every TMEM load has landed.
      auto release = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
      };

      if (!mbar_wait_bounded(&tfull[acc], acc_phase, abort_flag, status,
                             kStatusEpilogueTimeout, wait_limit)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (nchunks == 0) {
        release();
      } else {
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(32 * q) << 16) +
                               static_cast<uint32_t>(acc * BN + 32 * c_first);
        // TMEM loads run one chunk ahead of the math (two register sets), the
        // addend loads one chunk ahead as well.
        uint32_t va[32], vb[32];
        uint4 cv_next[4];
        load_addend(c_first, cv_next);
        tmem_ld_32x32b_x32_async(tbase, va);
        tmem_ld_wait_regs(va);
        if (nchunks == 1) release();
        for (int i = 0; i < nchunks; i += 2) {
          const int c = c_first + i;
          uint4 cva[4] = {cv_next[0], cv_next[1], cv_next[2], cv_next[3]};
          const bool has_b = i + 1 < nchunks;
          if (has_b) {
            load_addend(c + 1, cv_next);
            tmem_ld_32x32b_x32_async(tbase + 32 * (i + 1), vb);
          }
          process(c, va, cva);
          if (has_b) {
            tmem_ld_wait_regs(vb);
            if (i + 1 == nchunks - 1) release();
            uint4 cvb[4] = {cv_next[0], cv_next[1], cv_next[2], cv_next[3]};
            const bool has_a = i + 2 < nchunks;
            if (has_a) {
              load_addend(c + 2, cv_next);
              tmem_ld_32x32b_x32_async(tbase + 32 * (i + 2), va);
            }
            process(c + 1, vb, cvb);
            if (has_a) {
              tmem_ld_wait_regs(va);
              if (i + 2 == nchunks - 1) release();
            }
          }
        }
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait<0>();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

}  // namespace ps
