// CTA-pair (cta_group::2) version of the GEMM family of ps_gemm.cuh.
//
// Two CTAs of a cluster (an SM pair) compute one 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M = 256, N = 256): each CTA stages its own 128 rows
// of A and its own half (128 columns) of B, the leader CTA issues the UMMAs,
// and each CTA's TMEM receives its 128 x 256 accumulator. Against the 1-CTA
// kernel this halves the B bytes each SM streams from L2 and shrinks a stage
// to 32 KB, which leaves room for a 5-deep load ring and 8 epilogue warps
// (two per TMEM lane quarter, each draining 128 of the 256 columns).
//
// Symmetric products use 128-row blocks as before: a pair tile covers block
// rows 2q (leader) and 2q+1 (peer) against block columns 2p, 2p+1 for q <= p;
// a CTA stores a block it computed only if it lies on or above the diagonal,
// mirrored when strictly above (so each block pair still has one owner).
//
// Triangle storage (used inside a circuit): a symmetric result may be stored
// as its blocks on and above the diagonal only (store_mirror = 0), and an
// operand stored that way (a_tri / b_tri) is read back as a full matrix: a
// k-block whose 128x128 block lies below the diagonal is loaded from the
// stored transposed block with the other operand majorness (TMA box and UMMA
// descriptor switch per k-block). One instruction serves both CTAs' halves,
// so the pair switches together; it may then read a diagonal block
// transposed, which is exact because those blocks are bit-symmetric.
//
// Pipeline, per pair: both producers wait for their own free stage and load
// into their own shared memory, counting bytes on the leader's full barrier
// (the leader alone arms it with both CTAs' bytes); the leader's UMMA thread
// frees a stage in both CTAs and announces an accumulator to both epilogues
// with tcgen05.commit; all 16 epilogue warps release an accumulator on the
// leader's barrier. Every wait is bounded as in ps_gemm.cuh. Loads fill only
// the issuing CTA's own shared memory.
//
// Diagonal pair tiles of A . A^T (q == p, same_ab): each CTA's half of B is
// the same 128 rows as its A block, read through an identical map, so the
// producers load only A, the leader arms the barrier with A's bytes alone and
// the B descriptor points at the A stage. The UMMAs read the same bytes as
// with a separate B copy, so the results are unchanged, and these tiles stream
// half the operand bytes from L2.
#pragma once

#include <type_traits>

#include "ps_gemm.cuh"

namespace ps {
namespace pair {

constexpr int BM = 128;                 // rows per CTA
constexpr int BN = 256;                 // accumulator columns per CTA (pair N)
constexpr int BNH = 128;                // B columns staged per CTA
constexpr int BK = 128;                 // K per stage: two 64-wide (128-byte) sub-blocks
constexpr int STAGES = 3;
constexpr int UMMA_K = 16;
constexpr int SLAB_BYTES = 128 * 64 * 2;       // 16 KB: 128 rows (or K) x 64 halves
constexpr int A_STAGE_BYTES = BM * BK * 2;     // 32 KB
constexpr int B_STAGE_BYTES = BNH * BK * 2;    // 32 KB
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int NUM_EPI_WARPS = 8;
constexpr int NUM_THREADS = 64 + 32 * NUM_EPI_WARPS;  // 320
constexpr int EPI_WARP_BYTES = 4096;
constexpr int SMEM_OPERANDS = STAGES * STAGE_BYTES;
constexpr int SMEM_EPI = NUM_EPI_WARPS * EPI_WARP_BYTES;
constexpr int SMEM_CTRL = 256;
constexpr int SMEM_TOTAL = SMEM_OPERANDS + SMEM_EPI + SMEM_CTRL + 1024;
constexpr uint32_t TMEM_COLS = 2 * BN;
static_assert(SMEM_TOTAL <= 232448, "shared memory budget");

// One operand stage: 128 rows (or columns) of the operand by 128 of K, in
// two 16 KB slabs with 128-byte swizzle:
//   K-major : slab h = K sub-block h, [row 0..127][64 halves of K]
//   MN-major: slab j = 64-wide M/N half j, [k 0..127][64 halves of M/N]
// A "chunked" map (4-D: 64 | rows or K | 64-chunks | L) fills a stage with
// one TMA; a plain 3-D map takes two boxes (K-major) or four (MN-major). The
// per-instruction cost of a CTA-pair TMA, not its size, limits the operand
// stream, hence the large boxes.
__device__ __forceinline__ void load_operand(const CUtensorMap* map, bool chunked, bool mn_major,
                                             uint8_t* dst, uint32_t bar, int r0, int k0, int b) {
  if (!mn_major) {
    if (chunked) {
      tma_load_4d_pair(map, dst, bar, 0, r0, k0 / 64, b);
    } else {
      tma_load_3d_pair(map, dst, bar, k0, r0, b);
      tma_load_3d_pair(map, dst + SLAB_BYTES, bar, k0 + 64, r0, b);
    }
  } else {
    if (chunked) {
      tma_load_4d_pair(map, dst, bar, 0, k0, r0 / 64, b);
    } else {
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          tma_load_3d_pair(map, dst + j * SLAB_BYTES + h * (SLAB_BYTES / 2), bar, r0 + 64 * j,
                           k0 + 64 * h, b);
    }
  }
}

// Shared-memory descriptor pieces (tcgen05 format, 128-byte swizzle): the
// high word (stride between 8-row groups 1024 B, version 1, swizzle mode) is
// fixed; the low word holds the leading-byte offset and the start address.
constexpr uint32_t kDescHi = (1024u >> 4) | (1u << 14) | (2u << 29);
constexpr uint32_t kDescLoK = (16u >> 4) << 16;                               // K-major
constexpr uint32_t kDescLoMN = (static_cast<uint32_t>(SLAB_BYTES) >> 4) << 16;  // MN halves 16 KB apart

// The 8 UMMAs (2 sub-blocks x 4 of K = 16) of one stage.
__device__ __forceinline__ void mma_stage(uint32_t d_tmem, uint32_t a_addr, uint32_t b_addr,
                                          bool a_mn, bool b_mn, uint32_t idesc0, bool first) {
  const uint32_t idesc = idesc0 | (a_mn ? (1u << 15) : 0u) | (b_mn ? (1u << 16) : 0u);
  const uint32_t alo = (a_mn ? kDescLoMN : kDescLoK) | (a_addr >> 4);
  const uint32_t blo = (b_mn ? kDescLoMN : kDescLoK) | (b_addr >> 4);
  // per sub-block: MN-major 64 K-rows (8 KB), K-major one 16 KB slab; per
  // UMMA_K step: MN-major 16 K-rows (2 KB), K-major 32 bytes (>> 4 below)
  const uint32_t a_sub = a_mn ? 512u : 1024u, b_sub = b_mn ? 512u : 1024u;
  const uint32_t a_kk = a_mn ? 128u : 2u, b_kk = b_mn ? 128u : 2u;
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint64_t ad = (static_cast<uint64_t>(kDescHi) << 32) | (alo + h * a_sub + kk * a_kk);
      const uint64_t bd = (static_cast<uint64_t>(kDescHi) << 32) | (blo + h * b_sub + kk * b_kk);
      umma_f16_pair(d_tmem, ad, bd, idesc, (first && h == 0 && kk == 0) ? 0u : 1u);
    }
}

struct PairArgs {
  int M, N, K, L;
  int tiles_m2, tiles_n;  // general: pair tiles (256 rows) x column tiles
  int tb;                 // symmetric: 128-row blocks
  int tiles_per_mat, total_tiles;
  int group_m;            // general: pair-tile rows per rasterisation group
  float alpha, beta, diag;
  const __half* C;
  long long c_ld, c_bs;
  int has_addend, has_diag;
  int a_tri, b_tri;       // operand stored as upper-triangle blocks only
  int store_mirror;       // symmetric: also store the transposed off-diagonal blocks
  int same_ab;            // symmetric A . A^T, A and B maps identical (see below)
  int a_chunk, b_chunk, a2_chunk, b2_chunk;  // map is 4-D chunked (one TMA per stage)
  // General products only: instead of storing the result, apply it as a
  // Muon update to a parameter bank P (same layout as the output):
  // p <- fl(fl(p * decay) + upd_alpha * fl(u)), u the result in the output type.
  int upd, p_dtype;
  void* P;
  long long p_ld, p_bs;
  float decay, upd_alpha;
  int* status;
  long long wait_limit;
};

// The Muon update of one output row's 32 values (the FP32 epilogue values f,
// before the circuit's FP16 rounding) into row `row` of parameter matrix b of
// type T: u = OUT(fp16(f)) as the circuit would store it, then p <- fl_T(fma(
// alpha, fl_T(u), fl_T(p * decay))) as ps_muon_update_kernel computes it.
template <int OUT, typename T>
__device__ __forceinline__ void update_row_t(const PairArgs& a, int b, int row, int col0, int nv,
                                             const float (&f)[32]) {
  T* p = static_cast<T*>(a.P) + static_cast<long long>(b) * a.p_bs +
         static_cast<long long>(row) * a.p_ld + col0;
  auto rnd = [](float v) -> float {
    if (std::is_same<T, float>::value) return v;
    if (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(__float2bfloat16_rn(v));
    return __half2float(__float2half_rn(v));
  };
  auto to_f = [](T v) -> float {
    if constexpr (std::is_same<T, float>::value) return v;
    else if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(v);
    else return __half2float(v);
  };
  auto from_f = [](float v) -> T {
    if constexpr (std::is_same<T, float>::value) return v;
    else if constexpr (std::is_same<T, __nv_bfloat16>::value) return __float2bfloat16_rn(v);
    else return __float2half_rn(v);
  };
  constexpr int VW = 16 / sizeof(T);
  if (nv >= 32) {
#pragma unroll
    for (int v = 0; v < 32 / VW; ++v) {
      uint4 raw = ld_global_v4(p + v * VW);
      T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
      for (int i = 0; i < VW; ++i) {
        const int j = v * VW + i;
        float u = __half2float(__float2half_rn(f[j]));
        if (OUT == kOutBF16) u = __bfloat162float(__float2bfloat16_rn(u));
        const float w1 = rnd(__fmul_rn(to_f(e[i]), a.decay));
        e[i] = from_f(__fmaf_rn(a.upd_alpha, rnd(u), w1));
      }
      st_global_v4(p + v * VW, raw);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j >= nv) break;
      float u = __half2float(__float2half_rn(f[j]));
      if (OUT == kOutBF16) u = __bfloat162float(__float2bfloat16_rn(u));
      const float w1 = rnd(__fmul_rn(to_f(p[j]), a.decay));
      p[j] = from_f(__fmaf_rn(a.upd_alpha, rnd(u), w1));
    }
  }
}

template <bool SYM>
__device__ __forceinline__ void decode(const PairArgs& a, int t, uint32_t rank, int& b, int& m0,
                                       int& n0) {
  b = t / a.tiles_per_mat;
  int r = t - b * a.tiles_per_mat;
  if (SYM) {
    // column pair p owns row pairs 0..p
    int p = 0;
    while (r > p) {
      r -= p + 1;
      ++p;
    }
    m0 = (2 * r + static_cast<int>(rank)) * BM;
    n0 = 2 * p * BM;
  } else {
    const int per_group = a.group_m * a.tiles_n;
    const int g = r / per_group;
    const int first = g * a.group_m;
    const int gsz = min(a.group_m, a.tiles_m2 - first);
    const int idx = r - g * per_group;
    m0 = (first + idx % gsz) * (2 * BM) + static_cast<int>(rank) * BM;
    n0 = (idx / gsz) * BN;
  }
}

template <bool A_MN, bool B_MN, bool SYM, int OUT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    ps_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmA2,
                        const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmB2,
                        const __grid_constant__ CUtensorMap tmD, const PairArgs args) {
  // tmA / tmB: boxes in the operand's native majorness (A_MN / B_MN);
  // tmA2 / tmB2: the other majorness, used only for triangle-stored operands.
  constexpr bool kCanShare = SYM && (A_MN == B_MN);
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* s_epi = smem + SMEM_OPERANDS;
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_epi + SMEM_EPI);
  uint64_t* full = bars;                  // [STAGES] (used in the leader)
  uint64_t* empty = bars + STAGES;        // [STAGES]
  uint64_t* tfull = bars + 2 * STAGES;    // [2]
  uint64_t* tempty = tfull + 2;           // [2]   (used in the leader)
  uint64_t* drain = tempty + 2;           // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t peer = rank ^ 1u;
  const bool leader = rank == 0;
  const int pair_id = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
#pragma unroll
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * NUM_EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmD);
    if (args.a_tri) tma_prefetch_desc(&tmA2);
    if (args.b_tri) tma_prefetch_desc(&tmB2);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_kb = (args.K + BK - 1) / BK;
  const int ncols_total = args.N;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int t = pair_id; t < args.total_tiles && ok; t += npairs) {
        int b, m0, n0;
        decode<SYM>(args, t, rank, b, m0, n0);
        const int nb = n0 + static_cast<int>(rank) * BNH;  // this CTA's half of B
        const int a_lo = (m0 - static_cast<int>(rank) * BM) / BM;  // leader's row block
        const int b_lo = n0 / BM;                                 // leader's B block
        const bool share = kCanShare && args.same_ab && args.a_tri == args.b_tri && a_lo == b_lo;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, args.status,
                                 kStatusProducerTimeout, args.wait_limit)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = smem + stage * STAGE_BYTES;
          uint8_t* b_dst = a_dst + A_STAGE_BYTES;
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], share ? 2 * A_STAGE_BYTES : 2 * STAGE_BYTES);
          const int k0 = kb * BK;
          const bool at = args.a_tri && tri_transposed(A_MN, a_lo, a_lo + 1, k0 / BM);
          const bool bt = args.b_tri && tri_transposed(B_MN, b_lo, b_lo + 1, k0 / BM);
          load_operand(at ? &tmA2 : &tmA, (at ? args.a2_chunk : args.a_chunk) != 0, A_MN != at, a_dst,
                       bar, m0, k0, b);
          if (!share)  // a shared diagonal tile's B half is its A block: nothing more to load
            load_operand(bt ? &tmB2 : &tmB, (bt ? args.b2_chunk : args.b_chunk) != 0, B_MN != bt,
                         b_dst, bar, nb, k0, b);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Tail: every stage this CTA filled must have been released by the
      // leader's UMMAs (their commits arrive on this CTA's barriers) before
      // either CTA may exit.
      for (int s = 0; s < STAGES; ++s) {
        if (!(issued_mask & (1u << s))) continue;
        const uint32_t par = (issued_parity >> s) & 1u;
        const long long start = clock64();
        while (!mbar_try_wait(&empty[s], par)) {
          if (clock64() - start > args.wait_limit) {
            if (args.status) atomicCAS(args.status, 0, kStatusDrainTimeout);
            break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer (leader)
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued_any = false;

      const uint32_t empty_peer0 = mapa_shared(smem_u32(&empty[0]), peer);
      const uint32_t tfull_peer0 = mapa_shared(smem_u32(&tfull[0]), peer);
      const uint32_t smem_base = smem_u32(smem);
      const uint32_t idesc0 = make_idesc_f16(2 * BM, BN, false, false);
      for (int t = pair_id; t < args.total_tiles && ok; t += npairs) {
        if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1u, abort_flag, args.status,
                               kStatusMmaTimeout, args.wait_limit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        int tb_, tm0_, tn0_;
        decode<SYM>(args, t, 0, tb_, tm0_, tn0_);
        const int a_lo = tm0_ / BM, b_lo = tn0_ / BM;
        const bool share = kCanShare && args.same_ab && args.a_tri == args.b_tri && a_lo == b_lo;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, args.status, kStatusMmaTimeout,
                                 args.wait_limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_base + stage * STAGE_BYTES;
          const uint32_t b_addr = share ? a_addr : a_addr + A_STAGE_BYTES;
          const int kb128 = (kb * BK) / BM;
          const bool a_mn = A_MN != (args.a_tri && tri_transposed(A_MN, a_lo, a_lo + 1, kb128));
          const bool b_mn = B_MN != (args.b_tri && tri_transposed(B_MN, b_lo, b_lo + 1, kb128));
          mma_stage(d_tmem, a_addr, b_addr, a_mn, b_mn, idesc0, kb == 0);
          issued_any = true;
          // free this stage in both CTAs
          umma_commit_pair(smem_u32(&empty[stage]));
          umma_commit_pair(empty_peer0 + stage * 8);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&tfull[acc]));
        umma_commit_pair(tfull_peer0 + acc * 8);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok && issued_any) {
        umma_commit_pair(smem_u32(drain));
        const long long start = clock64();
        while (!mbar_try_wait(drain, 0)) {
          if (clock64() - start > args.wait_limit) {
            if (args.status) atomicCAS(args.status, 0, kStatusDrainTimeout);
            break;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    constexpr int OB = OutTraits<OUT>::kBytes;
    constexpr int ROW_BYTES = 32 * OB;
    constexpr int BUF_BYTES = 32 * ROW_BYTES;
    constexpr int SLOT_BYTES = SYM ? 2 * BUF_BYTES : BUF_BYTES;
    constexpr int NSLOT = EPI_WARP_BYTES / SLOT_BYTES;
    static_assert(NSLOT >= 1, "epilogue staging needs a slot");
    static_assert(!SYM || OUT == kOutF16, "symmetric products are stored in FP16");
    const int q = warp & 3;               // TMEM lane quarter
    const int h = (warp - 2) >> 2;        // column half of the 256-column accumulator
    const uint32_t stg = smem_u32(s_epi + (warp - 2) * EPI_WARP_BYTES);
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty[0]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    int slot = 0;
    bool ok = true;
    for (int t = pair_id; t < args.total_tiles && ok; t += npairs) {
      int b, m0, n0;
      decode<SYM>(args, t, rank, b, m0, n0);
      const int c_first = 4 * h;            // this warp's chunks: c_first .. c_first + 3
      int nvalid = ncols_total - (n0 + 32 * c_first);
      nvalid = nvalid > 128 ? 128 : nvalid;
      const int nchunks = nvalid > 0 ? (nvalid + 31) >> 5 : 0;
      const int row0 = m0 + 32 * q;
      const int grow = row0 + lane;
      // symmetric: skip blocks below the diagonal (another CTA owns their pair)
      const int blk_col = (n0 + 32 * c_first) / BM;
      const bool skip_block = SYM && (m0 / BM) > blk_col;
      const bool work = nchunks > 0 && !skip_block && row0 < args.M;
      const bool row_ok = grow < args.M;
      const bool load_c = work && args.has_addend && row_ok;
      const __half* crow =
          args.has_addend ? args.C + static_cast<long long>(b) * args.c_bs +
                                static_cast<long long>(grow) * args.c_ld
                          : nullptr;
      if (load_c) {
        const int cb = n0 + 32 * c_first;
        const int ce = min(cb + nvalid, ncols_total);
        for (int cc = cb; cc < ce; cc += 64) prefetch_l2(crow + cc);
        prefetch_l2(crow + ce - 1);
      }
      auto load_addend = [&](int c, uint4 (&dst)[4]) {
        const int g0 = n0 + 32 * c;
        if (!load_c) {
#pragma unroll
          for (int j = 0; j < 4; ++j) dst[j] = make_uint4(0, 0, 0, 0);
        } else if (g0 + 32 <= ncols_total) {
#pragma unroll
          for (int j = 0; j < 4; ++j) dst[j] = ld_global_v4(crow + g0 + 8 * j);
        } else {
          __half* hv = reinterpret_cast<__half*>(dst);
          for (int j = 0; j < 32; ++j)
            hv[j] = (g0 + j < ncols_total) ? crow[g0 + j] : __float2half(0.f);
        }
      };
      auto process = [&](int c, const uint32_t (&v)[32], const uint4 (&cv)[4]) {
        const int gcol0 = n0 + 32 * c;
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
        if (!SYM && args.upd) {
          if (grow < args.M) {
            const int nv = ncols_total - gcol0;
            if (args.p_dtype == kOutF32)
              update_row_t<OUT, float>(args, b, grow, gcol0, nv, f);
            else if (args.p_dtype == kOutBF16)
              update_row_t<OUT, __nv_bfloat16>(args, b, grow, gcol0, nv, f);
            else
              update_row_t<OUT, __half>(args, b, grow, gcol0, nv, f);
          }
          return;
        }
        uint32_t w[32];
        convert_row<OUT>(f, w);
        const bool mirror = SYM && args.store_mirror && (gcol0 / BM) != (m0 / BM);
        if (lane == 0) bulk_wait_read<NSLOT - 1>();
        __syncwarp();
        const uint32_t sb = stg + slot * SLOT_BYTES;
        if (ROW_BYTES == 64) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int p = j ^ ((lane >> 1) & 3);
            st_shared_v4(sb + lane * 64 + p * 16, w[4 * j], w[4 * j + 1], w[4 * j + 2],
                         w[4 * j + 3]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int p = j ^ (lane & 7);
            st_shared_v4(sb + lane * 128 + p * 16, w[4 * j], w[4 * j + 1], w[4 * j + 2],
                         w[4 * j + 3]);
          }
        }
        if (mirror) {
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
            tma_store_3d(&tmD, sb, gcol0, row0, b);
            if (mirror) tma_store_3d(&tmD, sb + BUF_BYTES, row0, gcol0, b);
          }
          bulk_commit();
        }
        slot = (slot + 1 == NSLOT) ? 0 : slot + 1;
      };
      auto release = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty_leader0 + acc * 8);
      };

      if (!mbar_wait_bounded(&tfull[acc], acc_phase, abort_flag, args.status,
                             kStatusEpilogueTimeout, args.wait_limit)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (!work) {
        release();
      } else {
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(32 * q) << 16) +
                               static_cast<uint32_t>(acc * BN + 32 * c_first);
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
  cluster_sync();  // neither CTA leaves while the other may still touch it
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, TMEM_COLS);
}

}  // namespace pair
}  // namespace ps
