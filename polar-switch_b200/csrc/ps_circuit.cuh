// A whole circuit in one persistent launch on CTA pairs: for every problem of
// a grouped call and every outer iteration t, the Gram B[0] = X X^T (X^T X
// when tall), the inner iterations B[w] = a B[i] B[i]^T + b B[r] + c I and
// the apply X' = B[last] X + delta X (X B[last] + delta X when tall), the
// last apply storing into the caller's output (or applying Muon's update to a
// parameter bank). Reference: polar_switch/__init__.py:40-44.
//
// Every tile is computed as the per-stage CTA-pair launches compute it (same
// operand views, stage layout, UMMA sequence and epilogue arithmetic), so the
// bits are those of ps_circuit_grouped's per-stage path. What changes is the
// schedule, as in ps_chain.cuh but across all stages: per matrix the stages
// form one chain G_0, S_0,0 .. S_0,k-1, A_0, G_1, ..., A_{T-1}, each reading
// what the previous one stored. Every epilogue warp publishes its part of a
// tile on its matrix's counter (stores waited for, proxy fence, release add);
// a tile of stage sigma waits (bounded) until the counter holds every part of
// every earlier stage of its matrix. The tile list is ordered in rounds over
// chunks of each problem's matrices (round r holds stage sigma of chunk
// r - sigma), so a wait is on tiles scheduled a round earlier. Dependencies
// point only to earlier tiles and each CTA walks its tiles in order; all CTAs
// of the grid are resident, so the earliest unfinished tile can always run.
#pragma once

#include "ps_chain.cuh"

namespace ps {
namespace circ {

constexpr int MAXP = 8;         // problems per launch
constexpr int MAXB = 3;         // square buffers
constexpr int MAX_STAGES = 48;  // stages per matrix (Gram, inner iterations, apply per outer)
constexpr int MAX_STEPS = 40;   // inner iterations over all outer iterations
constexpr int MAX_ITEMS = 768;  // (stage, problem, chunk) items
constexpr int MAX_PEERS = 7;    // other GPUs a final result is also stored to
constexpr int MAX_PHASES = 8;   // groups of matrices scheduled one after another
constexpr int SIGNALS_PER_TILE = 2 * pair::NUM_EPI_WARPS;

enum Kind : int { kGram = 0, kSquare = 1, kApply = 2 };

struct alignas(64) CProblem {
  // Xh[0], Xh[1] (Rp x Cp FP16): operand views (K-major, MN-major) and 32 x 32
  // output boxes; the square buffers (this problem's slice, n x n): operand
  // views and output boxes; the final output (y_out boxes).
  CUtensorMap xk[2], xm[2], xo[2];
  CUtensorMap bk[MAXB], bm[MAXB], bo[MAXB];
  CUtensorMap yo;
  const __half* xh[2];
  const __half* buf[MAXB];
  int L, Rp, Cp, n, m, tall;
  int Tsym, tiles_m2, tiles_n;    // pair tiles per matrix: symmetric, apply (M x N)
  int chunk, g0;                  // matrices per chunk; first matrix in the counter array
  int ck_x, ck_b;                 // X / buffer views are 4-D chunked maps
  int direct;                     // last apply stores into y (else into Xh)
  int y_out;                      // kOutF16 / kOutF32 / kOutBF16
  int upd, p_dtype;               // Muon update of P in place of storing y
  void* P;
  unsigned char* y;               // y (push: the local copy the peers' copies mirror)
  float decay, upd_alpha;
};

struct alignas(64) CircuitParams {
  CProblem prob[MAXP];
  chain::Step steps[MAX_STEPS];
  float residual[MAX_STAGES];     // per outer iteration
  // per stage: kind, outer iteration, step (square: its inner iteration; apply:
  // the last inner iteration of its outer iteration, whose buffer it uses),
  // and the symmetric / apply stages before it
  unsigned char st_kind[MAX_STAGES], st_t[MAX_STAGES], st_step[MAX_STAGES];
  unsigned char st_nsym[MAX_STAGES], st_napp[MAX_STAGES];
  int n_outer, n_stages, nprob;
  int n_items, total_tiles;
  unsigned* done;                 // per-matrix completion counters, zero at launch
  int* status;
  long long wait_limit;
  int item_start[MAX_ITEMS + 1];
  unsigned short item_first[MAX_ITEMS];  // first matrix (within its problem) of the item's chunk
  unsigned char item_stage[MAX_ITEMS], item_prob[MAX_ITEMS];
  // Push: every tile a final apply stores into y is also stored into n_peers
  // other GPUs' copies of y, at y + peer_delta[k] bytes (plain vector stores
  // of whole 16-byte granules, eight 64- or 128-byte row segments per warp
  // instruction). A final apply has no dependent stage, so pushed tiles are
  // not published on the counters; their stores complete by kernel exit.
  int n_peers;
  long long peer_delta[MAX_PEERS];
  // Phase signals (copy engines moving each phase's results while later
  // phases compute): sig[k] (k < n_sig) is set to 1 once every final-apply
  // tile of phase k is stored (sig[n_sig + k] counts their epilogue warps up
  // to sig_target[k]); sig[2 * n_sig] counts exiting CTAs, and the last one
  // sets every flag, so a wait on them always ends (after an abort too).
  // nullptr: off. The caller zeroes sig before the launch.
  unsigned* sig;
  int n_sig;
  unsigned sig_target[MAX_PHASES];
  unsigned char item_phase[MAX_ITEMS];
};
static_assert(sizeof(CircuitParams) <= 32764, "kernel parameter space");

struct Tile {
  int kind, p, b, t, s;  // stage kind, problem, matrix, outer iteration, step index
  int ph;                // phase of the tile's item
  int m0, n0;            // this CTA's first row; the pair's first column
  unsigned need;         // counter value the tile's inputs wait for (0: none)
};

__device__ __forceinline__ void decode(const CircuitParams& P, int t, uint32_t rank, Tile& d) {
  int lo = 0, hi = P.n_items - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (P.item_start[mid] <= t)
      lo = mid;
    else
      hi = mid - 1;
  }
  const int sg = P.item_stage[lo];
  const CProblem& q = P.prob[P.item_prob[lo]];
  d.p = P.item_prob[lo];
  d.ph = P.item_phase[lo];
  d.kind = P.st_kind[sg];
  d.t = P.st_t[sg];
  d.s = P.st_step[sg];
  const int per = d.kind == kApply ? q.tiles_m2 * q.tiles_n : q.Tsym;
  const int local = t - P.item_start[lo];
  const int mat = local / per;
  int r = local - mat * per;
  d.b = P.item_first[lo] + mat;
  d.need = sg == 0 ? 0u
                   : static_cast<unsigned>(SIGNALS_PER_TILE) *
                         (static_cast<unsigned>(P.st_nsym[sg]) * q.Tsym +
                          static_cast<unsigned>(P.st_napp[sg]) * (q.tiles_m2 * q.tiles_n));
  if (d.kind == kApply) {
    const int i = r / q.tiles_n, j = r - i * q.tiles_n;
    d.m0 = i * (2 * pair::BM) + static_cast<int>(rank) * pair::BM;
    d.n0 = j * pair::BN;
  } else {
    int pp = 0;
    while (r > pp) {
      r -= pp + 1;
      ++pp;
    }
    d.m0 = (2 * r + static_cast<int>(rank)) * pair::BM;
    d.n0 = 2 * pp * pair::BM;
  }
}

// The two operands of a tile: maps (native and transposed-block view), chunked
// flags, native majorness, triangle storage, K extent, diagonal sharing.
struct Operands {
  const CUtensorMap *a, *a2, *b, *b2;
  bool ack, a2ck, bck, b2ck;
  bool a_mn, b_mn, a_tri, b_tri, share;
  int K;
};

__device__ __forceinline__ void operands(const CircuitParams& P, const Tile& d, Operands& o) {
  const CProblem& q = P.prob[d.p];
  const int cur = d.t & 1;
  const bool ckx = q.ck_x != 0, ckb = q.ck_b != 0;
  const int a_lo = (d.m0 / pair::BM) & ~1, b_lo = d.n0 / pair::BM;
  if (d.kind == kGram) {
    // wide: X X^T from X's rows (K-major); tall: X^T X from its columns (MN-major)
    o.a = o.b = q.tall ? &q.xm[cur] : &q.xk[cur];
    o.a2 = o.b2 = o.a;
    o.ack = o.bck = o.a2ck = o.b2ck = ckx;
    o.a_mn = o.b_mn = q.tall != 0;
    o.a_tri = o.b_tri = false;
    o.share = a_lo == b_lo;
    o.K = q.m;
  } else if (d.kind == kSquare) {
    const int src = P.steps[d.s].src;
    o.a = o.b = &q.bk[src];
    o.a2 = o.b2 = &q.bm[src];
    o.ack = o.bck = o.a2ck = o.b2ck = ckb;
    o.a_mn = o.b_mn = false;
    o.a_tri = o.b_tri = true;
    o.share = a_lo == b_lo;
    o.K = q.n;
  } else {
    const int last = P.steps[d.s].dst;  // the buffer of the last inner iteration
    o.share = false;
    o.K = q.n;
    if (!q.tall) {  // B X: A = B[last] (K-major, triangle-stored), B = X read MN-major
      o.a = &q.bk[last];
      o.a2 = &q.bm[last];
      o.ack = o.a2ck = ckb;
      o.a_mn = false;
      o.a_tri = true;
      o.b = o.b2 = &q.xm[cur];
      o.bck = o.b2ck = ckx;
      o.b_mn = true;
      o.b_tri = false;
    } else {        // X B: A = X (K-major), B = B[last] read MN-major (triangle-stored)
      o.a = o.a2 = &q.xk[cur];
      o.ack = o.a2ck = ckx;
      o.a_mn = false;
      o.a_tri = false;
      o.b = &q.bm[last];
      o.b2 = &q.bk[last];
      o.bck = o.b2ck = ckb;
      o.b_mn = true;
      o.b_tri = true;
    }
  }
}

// A tile's epilogue values (the FP32 accumulator column chunk of one row,
// after alpha/beta/diag) converted and staged for the TMA store, by output
// type (FP16 and BF16: 64-byte rows with 64-byte swizzle; FP32: 128-byte rows
// with 128-byte swizzle, the maps' swizzles).
template <int OUT>
__device__ __forceinline__ void stage_row(uint32_t sb, int lane, const float (&f)[32]) {
  uint32_t w[32];
  convert_row<OUT>(f, w);
  if (OutTraits<OUT>::kBytes == 2) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int p = j ^ ((lane >> 1) & 3);
      st_shared_v4(sb + lane * 64 + p * 16, w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int p = j ^ (lane & 7);
      st_shared_v4(sb + lane * 128 + p * 16, w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
    }
  }
}

// The staged 32-row box (stage_row's layout) stored into every peer's copy
// of y with 16-byte stores: lane l reads granule l % G of row l / G (G
// granules per row), so one warp instruction writes 32 / G whole row
// segments; the registers are reused for every peer. Rows at or beyond M and
// granules at or beyond N (a multiple of 8 columns) are skipped.
__device__ __noinline__ void push_box(const CircuitParams& P, unsigned char* y, int out,
                                         uint32_t sb, int lane, int b, int row0, int gcol0, int M,
                                         int N) {
  const int eb = out == kOutF32 ? 4 : 2;           // element bytes
  const int G = eb == 4 ? 8 : 4;                   // 16-byte granules per staged row
  const int rows_per = 32 / G;
  const int j = lane % G;
  const int col = gcol0 + j * (16 / eb);
#pragma unroll 1
  for (int r0 = 0; r0 < 32; r0 += rows_per) {
    const int r = r0 + lane / G;
    const int p = eb == 4 ? (j ^ (r & 7)) : (j ^ ((r >> 1) & 3));
    uint32_t a, bb, c, dd;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(a), "=r"(bb), "=r"(c), "=r"(dd)
                 : "r"(sb + r * (G * 16) + p * 16));
    const int row = row0 + r;
    if (row < M && col < N) {
      const long long off = ((static_cast<long long>(b) * M + row) * N + col) * eb;
      for (int k = 0; k < P.n_peers; ++k) {
        unsigned char* dst = y + off + P.peer_delta[k];
        asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "r"(a), "r"(bb), "r"(c),
                     "r"(dd)
                     : "memory");
      }
    }
  }
}

__global__ void __launch_bounds__(pair::NUM_THREADS, 1)
    ps_circuit_pair_kernel(const __grid_constant__ CircuitParams P) {
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
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      int ready_g = -1;
      unsigned ready_need = 0;
      for (int t = pair_id; t < P.total_tiles && ok; t += npairs) {
        Tile d;
        decode(P, t, rank, d);
        const int g = P.prob[d.p].g0 + d.b;
        if (d.need && !(g == ready_g && d.need <= ready_need)) {
          // every earlier stage of this matrix must be stored before it is read
          if (!counter_wait_bounded(P.done + g, d.need, abort_flag, P.status,
                                    kStatusDependencyTimeout, P.wait_limit)) {
            ok = false;
            break;
          }
          fence_proxy_async_global();
          ready_g = g;
          ready_need = d.need;
        }
        Operands o;
        operands(P, d, o);
        const int num_kb = (o.K + BK - 1) / BK;
        const int nb = d.n0 + static_cast<int>(rank) * BNH;          // this CTA's half of B
        const int a_lo = (d.m0 - static_cast<int>(rank) * BM) / BM;  // leader's row block
        const int b_lo = d.n0 / BM;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, P.status,
                                 kStatusProducerTimeout, P.wait_limit)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = smem + stage * STAGE_BYTES;
          uint8_t* b_dst = a_dst + A_STAGE_BYTES;
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&full[stage], o.share ? 2 * A_STAGE_BYTES : 2 * STAGE_BYTES);
          const int k0 = kb * BK;
          const bool at = o.a_tri && tri_transposed(o.a_mn, a_lo, a_lo + 1, k0 / BM);
          const bool bt = o.b_tri && tri_transposed(o.b_mn, b_lo, b_lo + 1, k0 / BM);
          pair::load_operand(at ? o.a2 : o.a, at ? o.a2ck : o.ack, o.a_mn != at, a_dst, bar, d.m0, k0,
                             d.b);
          if (!o.share)
            pair::load_operand(bt ? o.b2 : o.b, bt ? o.b2ck : o.bck, o.b_mn != bt, b_dst, bar, nb, k0,
                               d.b);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
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
        Tile d;
        decode(P, t, 0, d);
        Operands o;
        operands(P, d, o);
        const int num_kb = (o.K + BK - 1) / BK;
        const int a_lo = d.m0 / BM, b_lo = d.n0 / BM;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, P.status, kStatusMmaTimeout,
                                 P.wait_limit)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_base + stage * STAGE_BYTES;
          const uint32_t b_addr = o.share ? a_addr : a_addr + A_STAGE_BYTES;
          const int kb128 = (kb * BK) / BM;
          const bool a_mn = o.a_mn != (o.a_tri && tri_transposed(o.a_mn, a_lo, a_lo + 1, kb128));
          const bool b_mn = o.b_mn != (o.b_tri && tri_transposed(o.b_mn, b_lo, b_lo + 1, kb128));
          pair::mma_stage(d_tmem, a_addr, b_addr, a_mn, b_mn, idesc0, kb == 0);
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
    const int q4 = warp & 3;              // TMEM lane quarter
    const int h = (warp - 2) >> 2;        // column half of the 256-column accumulator
    const uint32_t stg = smem_u32(s_epi + (warp - 2) * EPI_WARP_BYTES);
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty[0]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    int slot = 0;
    bool ok = true;
    for (int t = pair_id; t < P.total_tiles && ok; t += npairs) {
      Tile d;
      decode(P, t, rank, d);
      const CProblem& q = P.prob[d.p];
      const bool sym = d.kind != kApply;
      const bool final_apply = d.kind == kApply && d.t == P.n_outer - 1;
      const int cur = d.t & 1;
      // output: rows M x columns N, its map, type and addend
      const int M = sym ? q.n : (q.tall ? q.m : q.n);
      const int N = sym ? q.n : (q.tall ? q.n : q.m);
      int out = kOutF16;
      const CUtensorMap* tmD;
      const __half* C = nullptr;
      long long c_ld = 0, c_bs = 0;
      float alpha = 1.f, beta = 0.f, diag = 0.f;
      if (d.kind == kGram) {
        tmD = &q.bo[0];
      } else if (d.kind == kSquare) {
        const chain::Step& st = P.steps[d.s];
        tmD = &q.bo[st.dst];
        C = q.buf[st.add];
        c_ld = q.n;
        c_bs = static_cast<long long>(q.n) * q.n;
        alpha = st.alpha;
        beta = st.beta;
        diag = st.diag;
      } else {
        const float res = P.residual[d.t];
        if (res != 0.f) {
          C = q.xh[cur];
          c_ld = q.Cp;
          c_bs = static_cast<long long>(q.Rp) * q.Cp;
          beta = res;
        }
        if (final_apply && q.direct) {
          tmD = &q.yo;
          out = q.y_out;
        } else {
          tmD = &q.xo[1 - cur];
        }
      }
      const bool upd = final_apply && q.direct && q.upd;
      const bool push = final_apply && q.direct && !q.upd && P.n_peers > 0;
      const int c_first = 4 * h;
      int nvalid = N - (d.n0 + 32 * c_first);
      nvalid = nvalid > 128 ? 128 : nvalid;
      const int nchunks = nvalid > 0 ? (nvalid + 31) >> 5 : 0;
      const int row0 = d.m0 + 32 * q4;
      const int grow = row0 + lane;
      const int blk_col = (d.n0 + 32 * c_first) / BM;
      const bool skip_block = sym && (d.m0 / BM) > blk_col;  // triangle storage
      const bool work = nchunks > 0 && !skip_block && row0 < M;
      const bool load_c = work && C != nullptr && grow < M;
      const __half* crow = C ? C + d.b * c_bs + static_cast<long long>(grow) * c_ld : nullptr;
      // The addend was stored by an earlier stage of this matrix: lane 0
      // acquires its completion count for the warp.
      int seen = 1;
      if (lane == 0 && d.need && load_c)
        seen = counter_wait_bounded(P.done + q.g0 + d.b, d.need, abort_flag, P.status,
                                    kStatusDependencyTimeout, P.wait_limit);
      if (!__shfl_sync(0xffffffffu, seen, 0)) {
        ok = false;
        break;
      }
      if (load_c) {
        const int cb = d.n0 + 32 * c_first;
        const int ce = min(cb + nvalid, N);
        for (int cc = cb; cc < ce; cc += 64) prefetch_l2(crow + cc);
        prefetch_l2(crow + ce - 1);
      }
      auto load_addend = [&](int c, uint4 (&dst)[4]) {
        const int g0c = d.n0 + 32 * c;
        if (!load_c) {
#pragma unroll
          for (int j = 0; j < 4; ++j) dst[j] = make_uint4(0, 0, 0, 0);
        } else if (g0c + 32 <= N) {
#pragma unroll
          for (int j = 0; j < 4; ++j) dst[j] = ld_global_v4(crow + g0c + 8 * j);
        } else {
          __half* hv = reinterpret_cast<__half*>(dst);
          for (int j = 0; j < 32; ++j) hv[j] = (g0c + j < N) ? crow[g0c + j] : __float2half(0.f);
        }
      };
      auto process = [&](int c, const uint32_t (&v)[32], const uint4 (&cv)[4]) {
        const int gcol0 = d.n0 + 32 * c;
        float f[32];
        if (C) {
          const __half* hv = reinterpret_cast<const __half*>(cv);
#pragma unroll
          for (int j = 0; j < 32; ++j)
            f[j] = fmaf(beta, __half2float(hv[j]), alpha * __uint_as_float(v[j]));
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) f[j] = alpha * __uint_as_float(v[j]);
        }
        if (sym && diag != 0.f) {
          const int dd = grow - gcol0;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j == dd) f[j] += diag;
        }
        if (upd) {
          if (grow < M) {
            pair::PairArgs ua;
            ua.P = q.P;
            ua.p_ld = q.Cp;
            ua.p_bs = static_cast<long long>(q.Rp) * q.Cp;
            ua.decay = q.decay;
            ua.upd_alpha = q.upd_alpha;
            const int nv = N - gcol0;
            if (out == kOutF32) {
              if (q.p_dtype == kOutF32) pair::update_row_t<kOutF32, float>(ua, d.b, grow, gcol0, nv, f);
              else if (q.p_dtype == kOutBF16) pair::update_row_t<kOutF32, __nv_bfloat16>(ua, d.b, grow, gcol0, nv, f);
              else pair::update_row_t<kOutF32, __half>(ua, d.b, grow, gcol0, nv, f);
            } else if (out == kOutBF16) {
              if (q.p_dtype == kOutF32) pair::update_row_t<kOutBF16, float>(ua, d.b, grow, gcol0, nv, f);
              else if (q.p_dtype == kOutBF16) pair::update_row_t<kOutBF16, __nv_bfloat16>(ua, d.b, grow, gcol0, nv, f);
              else pair::update_row_t<kOutBF16, __half>(ua, d.b, grow, gcol0, nv, f);
            } else {
              if (q.p_dtype == kOutF32) pair::update_row_t<kOutF16, float>(ua, d.b, grow, gcol0, nv, f);
              else if (q.p_dtype == kOutBF16) pair::update_row_t<kOutF16, __nv_bfloat16>(ua, d.b, grow, gcol0, nv, f);
              else pair::update_row_t<kOutF16, __half>(ua, d.b, grow, gcol0, nv, f);
            }
          }
          return;
        }
        // FP32 rows fill a whole 4 KB slot; 16-bit rows half of one.
        const int slot_bytes = out == kOutF32 ? 4096 : 2048;
        if (lane == 0) {
          if (slot_bytes == 4096)
            bulk_wait_read<0>();
          else
            bulk_wait_read<1>();
        }
        __syncwarp();
        const uint32_t sb = stg + (slot_bytes == 4096 ? 0u : static_cast<uint32_t>(slot) * 2048u);
        if (out == kOutF32)
          stage_row<kOutF32>(sb, lane, f);
        else if (out == kOutBF16)
          stage_row<kOutBF16>(sb, lane, f);
        else
          stage_row<kOutF16>(sb, lane, f);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (row0 < M && gcol0 < N) {
            tma_store_3d(tmD, sb, gcol0, row0, d.b);
          }
          bulk_commit();
        }
        if (push) push_box(P, q.y, out, sb, lane, d.b, row0, gcol0, M, N);
        slot = (slot_bytes == 4096) ? 0 : (slot ^ 1);
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
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(32 * q4) << 16) +
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
      // Publish this warp's part of the tile (stores complete and visible);
      // pushed final tiles have no reader in this launch. A final tile of a
      // signalled launch also counts towards its phase, whose flag the last
      // of its warps raises (system scope: a copy engine reads the data).
      if (lane == 0 && !push) {
        bulk_wait<0>();
        fence_proxy_async_global();
        red_release_gpu_add_u32(P.done + q.g0 + d.b, 1u);
        if (final_apply && P.sig) {
          // GPU-scope acquire-release count (the stores are complete and
          // fenced above); the last warp of the phase, having acquired every
          // other warp's part, raises the flag with a system-scope release.
          const unsigned prev = atom_acq_rel_gpu_add_u32(P.sig + P.n_sig + d.ph, 1u);
          if (prev + 1 == P.sig_target[d.ph]) st_release_sys_u32(P.sig + d.ph, 1u);
        }
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
  if (P.sig && threadIdx.x == 0) {
    __threadfence_system();
    if (atomicAdd(P.sig + 2 * P.n_sig, 1u) == gridDim.x - 1)
      for (int k = 0; k < P.n_sig; ++k) st_release_sys_u32(P.sig + k, 1u);
  }
  cluster_sync();  // neither CTA leaves while the other may still touch it
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, TMEM_COLS);
}

}  // namespace circ
}  // namespace ps
