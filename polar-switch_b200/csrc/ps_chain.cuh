// All inner iterations of one outer iteration of a circuit in one persistent
// launch on CTA pairs ("chain"): B[dst_s] = alpha_s B[src_s] B[src_s]^T +
// beta_s B[add_s] + diag_s I for s = 0..S-1, over L stacked n x n matrices
// held as upper-triangle blocks (the circuit's square buffers).
//
// Each pair tile is computed exactly as ps_gemm_pair_kernel computes a square
// of triangle-stored buffers (same tiles, same UMMA sequence, same FP32
// epilogue and single FP16 rounding), so the results are the bits of S
// separate launches. What changes is the schedule:
//
//   * one tile list covers every (step, matrix, pair tile); step s of matrix
//     b may start once every tile of step s-1 of matrix b is stored. Each
//     epilogue warp publishes its part of a tile on a per-matrix counter
//     (its TMA stores waited for, a proxy fence, a release add), and a
//     producer about to load a tile of step s >= 1 waits (bounded) until the
//     counter says step s-1 of its matrix is complete;
//   * the list is ordered in rounds over chunks of matrices: round r holds
//     step s of chunk r - s for every s, so a chunk's buffers are reused by
//     the next step about S chunks later, while they are still in L2, and the
//     tile a producer waits for was scheduled S chunks of tiles earlier.
//
// Dependencies only point to earlier tiles and every CTA walks its tiles in
// order, so the earliest unfinished tile can always proceed; all CTAs of the
// grid are resident (one per SM, grid sized from the occupancy query). A wait
// that runs out records kStatusDependencyTimeout and the kernel returns early
// (the bounded-wait machinery of ps_gemm2.cuh). Reference behaviour: the
// inner loop of polar_switch/__init__.py:42-43.
#pragma once

#include "ps_gemm2.cuh"

namespace ps {
namespace chain {

constexpr int MAX_STEPS = 8;
constexpr int MAX_BUFS = 4;
constexpr int MAX_ITEMS = 512;
// Completion signals per pair tile: one per epilogue warp of both CTAs.
constexpr int SIGNALS_PER_TILE = 2 * pair::NUM_EPI_WARPS;

struct Step {
  int dst, src, add;
  float alpha, beta, diag;
};

struct alignas(64) ChainParams {
  CUtensorMap tmK[MAX_BUFS];   // K-major operand stages (see pair::load_operand)
  CUtensorMap tmMN[MAX_BUFS];  // MN-major operand stages: blocks read transposed
  CUtensorMap tmD[MAX_BUFS];   // 32 x 32 output boxes
  const __half* buf[MAX_BUFS]; // buffer bases: L stacked n x n matrices each
  Step steps[MAX_STEPS];
  int n, L;
  int T;                       // pair tiles per matrix
  int chunk;                   // matrices per chunk
  int n_items, total_tiles;
  int nbufs;
  int chunked;                 // tmK / tmMN are 4-D chunked maps (n % 64 == 0)
  unsigned base;               // counter value at the start of this launch
  unsigned* done;              // per-matrix completion counters
  int* status;
  long long wait_limit;        // cycles before an mbarrier wait gives up
  long long dep_limit;         // cycles before a wait on another tile's counter gives up
  int item_start[MAX_ITEMS + 1];  // first tile of each (step, chunk) item
  unsigned short item_step[MAX_ITEMS];
  unsigned short item_chunk[MAX_ITEMS];
};

// Tile t -> step s, matrix b, and this CTA's row offset m0 / the pair's column
// offset n0 (column pair p owns row pairs 0..p, as in ps_gemm2.cuh).
__device__ __forceinline__ void decode(const ChainParams& P, int t, uint32_t rank, int& s, int& b,
                                       int& m0, int& n0) {
  int lo = 0, hi = P.n_items - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (P.item_start[mid] <= t)
      lo = mid;
    else
      hi = mid - 1;
  }
  const int local = t - P.item_start[lo];
  s = P.item_step[lo];
  const int mat = local / P.T;
  int r = local - mat * P.T;
  b = P.item_chunk[lo] * P.chunk + mat;
  int p = 0;
  while (r > p) {
    r -= p + 1;
    ++p;
  }
  m0 = (2 * r + static_cast<int>(rank)) * pair::BM;
  n0 = 2 * p * pair::BM;
}

__global__ void __launch_bounds__(pair::NUM_THREADS, 1)
    ps_chain_pair_kernel(const __grid_constant__ ChainParams P) {
  // the CTA-pair tiling of ps_gemm2.cuh (these hide the one-CTA constants of ps::)
  using pair::A_STAGE_BYTES;
  using pair::BK;
  using pair::BM;
  using pair::BN;
  using pair::BNH;
  using pair::EPI_WARP_BYTES;
  using pair::NUM_EPI_WARPS;
  using pair::SMEM_EPI;
  using pair::SMEM_OPERANDS;
  using pair::STAGE_BYTES;
  using pair::STAGES;
  using pair::TMEM_COLS;
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
    for (int k = 0; k < P.nbufs; ++k) {
      tma_prefetch_desc(&P.tmK[k]);
      tma_prefetch_desc(&P.tmMN[k]);
      tma_prefetch_desc(&P.tmD[k]);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_kb = (P.n + BK - 1) / BK;
  const int ncols_total = P.n;
  const unsigned per_step = static_cast<unsigned>(SIGNALS_PER_TILE * P.T);

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      int ready_b = -1, ready_s = -1;
      for (int t = pair_id; t < P.total_tiles && ok; t += npairs) {
        int s, b, m0, n0;
        decode(P, t, rank, s, b, m0, n0);
        if (s > 0 && !(b == ready_b && s <= ready_s)) {
          // step s - 1 of matrix b must be stored before its buffer is read
          if (!counter_wait_bounded(P.done + b, P.base + static_cast<unsigned>(s) * per_step,
                                    abort_flag, P.status, kStatusDependencyTimeout, P.dep_limit)) {
            ok = false;
            break;
          }
          fence_proxy_async_global();
          ready_b = b;
          ready_s = s;
        }
        const int src = P.steps[s].src;
        const CUtensorMap* mk = &P.tmK[src];
        const CUtensorMap* mmn = &P.tmMN[src];
        const int nb = n0 + static_cast<int>(rank) * BNH;          // this CTA's half of B
        const int a_lo = (m0 - static_cast<int>(rank) * BM) / BM;  // leader's row block
        const int b_lo = n0 / BM;                                  // leader's B block
        const bool share = a_lo == b_lo;  // diagonal pair tile: B half == A block
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, P.status,
                                 kStatusProducerTimeout, P.wait_limit)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = smem + stage * STAGE_BYTES;
          uint8_t* b_dst = a_dst + A_STAGE_BYTES;
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], share ? 2 * A_STAGE_BYTES : 2 * STAGE_BYTES);
          const int k0 = kb * BK;
          const bool at = tri_transposed(false, a_lo, a_lo + 1, k0 / BM);
          const bool bt = tri_transposed(false, b_lo, b_lo + 1, k0 / BM);
          pair::load_operand(at ? mmn : mk, P.chunked != 0, at, a_dst, bar, m0, k0, b);
          if (!share)  // diagonal pair tile: B half == A block
            pair::load_operand(bt ? mmn : mk, P.chunked != 0, bt, b_dst, bar, nb, k0, b);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Every stage this CTA filled must have been released by the leader's
      // UMMAs before either CTA may exit.
      for (int s = 0; s < STAGES; ++s) {
        if (!(issued_mask & (1u << s))) continue;
        const uint32_t par = (issued_parity >> s) & 1u;
        const long long start = clock64();
        while (!mbar_try_wait(&empty[s], par)) {
          if (clock64() - start > P.wait_limit) {
            if (P.status) atomicCAS(P.status, 0, kStatusDrainTimeout);
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
      for (int t = pair_id; t < P.total_tiles && ok; t += npairs) {
        if (!mbar_wait_bounded(&tempty[acc], acc_phase ^ 1u, abort_flag, P.status,
                               kStatusMmaTimeout, P.wait_limit)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        int s_, b_, tm0, tn0;
        decode(P, t, 0, s_, b_, tm0, tn0);
        const int a_lo = tm0 / BM, b_lo = tn0 / BM;
        const bool share = a_lo == b_lo;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, P.status, kStatusMmaTimeout,
                                 P.wait_limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_base + stage * STAGE_BYTES;
          const uint32_t b_addr = share ? a_addr : a_addr + A_STAGE_BYTES;
          const int kb128 = (kb * BK) / BM;
          pair::mma_stage(d_tmem, a_addr, b_addr, tri_transposed(false, a_lo, a_lo + 1, kb128),
                          tri_transposed(false, b_lo, b_lo + 1, kb128), idesc0, kb == 0);
          issued_any = true;
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
          if (clock64() - start > P.wait_limit) {
            if (P.status) atomicCAS(P.status, 0, kStatusDrainTimeout);
            break;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    constexpr int ROW_BYTES = 64;                 // 32 FP16 values
    constexpr int BUF_BYTES = 32 * ROW_BYTES;     // one 32 x 32 sub-tile
    constexpr int NSLOT = EPI_WARP_BYTES / BUF_BYTES;
    const int q = warp & 3;               // TMEM lane quarter
    const int h = (warp - 2) >> 2;        // column half of the 256-column accumulator
    const uint32_t stg = smem_u32(s_epi + (warp - 2) * EPI_WARP_BYTES);
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty[0]), 0);
    const long long nn = static_cast<long long>(P.n) * P.n;
    int acc = 0;
    uint32_t acc_phase = 0;
    int slot = 0;
    bool ok = true;
    for (int t = pair_id; t < P.total_tiles && ok; t += npairs) {
      int s, b, m0, n0;
      decode(P, t, rank, s, b, m0, n0);
      const Step& st = P.steps[s];
      const int c_first = 4 * h;            // this warp's chunks: c_first .. c_first + 3
      int nvalid = ncols_total - (n0 + 32 * c_first);
      nvalid = nvalid > 128 ? 128 : nvalid;
      const int nchunks = nvalid > 0 ? (nvalid + 31) >> 5 : 0;
      const int row0 = m0 + 32 * q;
      const int grow = row0 + lane;
      // blocks below the diagonal are not stored (triangle storage)
      const int blk_col = (n0 + 32 * c_first) / BM;
      const bool skip_block = (m0 / BM) > blk_col;
      const bool work = nchunks > 0 && !skip_block && row0 < P.n;
      const bool load_c = work && grow < P.n;
      const __half* crow = P.buf[st.add] + b * nn + static_cast<long long>(grow) * P.n;
      // The addend was stored by an earlier step of this matrix; the producer
      // of this tile has seen that, this warp makes sure of it for itself
      // (lane 0 acquires, __syncwarp orders the other lanes' loads after it).
      int seen = 1;
      if (lane == 0 && s > 0 && work)
        seen = counter_wait_bounded(P.done + b, P.base + static_cast<unsigned>(s) * per_step,
                                    abort_flag, P.status, kStatusDependencyTimeout, P.dep_limit);
      seen = __shfl_sync(0xffffffffu, seen, 0);
      if (!seen) {
        ok = false;
        break;
      }
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
        const __half* hv = reinterpret_cast<const __half*>(cv);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          f[j] = fmaf(st.beta, __half2float(hv[j]), st.alpha * __uint_as_float(v[j]));
        if (st.diag != 0.f) {
          const int d = grow - gcol0;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j == d) f[j] += st.diag;
        }
        uint32_t w[32];
        convert_row<kOutF16>(f, w);
        if (lane == 0) bulk_wait_read<NSLOT - 1>();
        __syncwarp();
        const uint32_t sb = stg + slot * BUF_BYTES;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int p = j ^ ((lane >> 1) & 3);
          st_shared_v4(sb + lane * 64 + p * 16, w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (row0 < P.n && gcol0 < ncols_total) tma_store_3d(&P.tmD[st.dst], sb, gcol0, row0, b);
          bulk_commit();
        }
        slot = (slot + 1 == NSLOT) ? 0 : slot + 1;
      };
      auto release = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty_leader0 + acc * 8);
      };

      if (!mbar_wait_bounded(&tfull[acc], acc_phase, abort_flag, P.status,
                             kStatusEpilogueTimeout, P.wait_limit)) {
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
      // Publish this warp's part of the tile: its stores are complete and
      // visible before the count that later steps of matrix b wait for.
      if (lane == 0) {
        bulk_wait<0>();
        fence_proxy_async_global();
        red_release_gpu_add_u32(P.done + b, 1u);
      }
      __syncwarp();
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

}  // namespace chain
}  // namespace ps
