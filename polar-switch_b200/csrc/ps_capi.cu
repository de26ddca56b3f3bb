// C-ABI entry points of libpolarswitch_b200.so: argument validation, TMA
// tensor-map encoding, launch configuration and the circuit driver. One
// translation unit holds all device code so the status word is a single
// module-scope symbol.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "../../include/polar_switch_b200.h"
#include "ps_gemm.cuh"
#include "ps_gemm2.cuh"
#include "ps_chain.cuh"
#include "ps_circuit.cuh"
#include "ps_norm.cuh"
#include "ps_muon.cuh"
#include "ps_stats.cuh"

namespace ps {
// First error code recorded by a bounded wait in any kernel on this device.
__device__ int g_status;

// Scratch of ps_normalize_noalloc: the per-chunk sums of squares of pass 1,
// PS_NORMALIZE_NOALLOC_MAX_PARTIALS doubles (256 KiB). It lives in the
// library's module, so every GPU that loads the library holds it until the
// process exits, and every call of ps_normalize_noalloc on a device shares it.
static __device__ __align__(256) double g_noalloc_partials[PS_NORMALIZE_NOALLOC_MAX_PARTIALS];
}  // namespace ps

namespace {

constexpr int kVersion = 100;  // 0.1.0
constexpr int kMaxDevices = 64;
constexpr int kNumVariants = 16;

// Launch classes reported by ps_profile_read.
enum ProfKind : int {
  kProfNormalize = 0,
  kProfGram = 1,
  kProfSquare = 2,
  kProfApply = 3,
  kProfOther = 4,
  kProfCircuit = 5,  // whole circuits in one launch (ps_circuit.cuh)
  kNumProfKinds = 6
};

thread_local std::string g_last_error;
long long g_wait_limit = ps::kDefaultWaitLimit;
// Which GEMM kernel runs: 0 = the one-CTA kernel, 1 (default) = the CTA-pair
// kernel for every product, 2 = CTA pairs for squares of buffers up to
// kPairMaxN and the one-CTA kernel for everything else. With whole 128-wide K
// stages per TMA the pair kernel measured faster than or equal to mode 2 on
// every BASELINE workload (Qwen step +4 %, 8192^2 circuit +8 %).
int g_pair_mode = 1;
constexpr int64_t kPairMaxN = 1024;
// Upper bound on the CTAs (SMs) a persistent GEMM grid may take; 0 = all SMs.
// Leaving SMs free lets a collective run beside the GEMMs.
int g_max_ctas = 0;
// Inner iterations of a grouped circuit on the CTA-pair path run as one
// persistent chain launch per outer iteration (1, default) or one launch per
// inner iteration (0). Both give the same bits.
int g_chain_mode = 1;
// A grouped circuit on the CTA-pair path runs as one persistent launch for all
// its stages (1, default) or one launch per stage (0). Same bits either way;
// measured equal on the 196-matrix Qwen step and 1.6x faster on its 25-matrix
// share of one rank at 8 GPUs (2x on one 7-matrix layer).
int g_circuit_mode = 1;
// Normalisations of grouped circuits read each contiguous input once (the
// fused single-read kernel) when 1, or run the two passes when 0 (default).
// Both give the same bits; the single read measured slower on the Qwen step
// (2.7 against 6.2 TB/s of algorithmic traffic: CTAs holding chunks wait for
// the rest of their matrix in waves), so it is off until that is fixed.
int g_norm_fused = 0;

// Every kernel launch of the library is counted; when profiling is enabled,
// each launch is also bracketed by CUDA events on its stream and tagged with
// its algorithmic FLOPs and bytes.
std::atomic<long long> g_launches{0};

struct ProfRecord {
  int kind;
  cudaEvent_t start, stop;
  double flops, bytes;
};
std::mutex g_prof_mu;
bool g_prof_on = false;
std::vector<ProfRecord> g_prof;
std::vector<cudaEvent_t> g_event_pool;

cudaEvent_t pooled_event() {
  if (!g_event_pool.empty()) {
    cudaEvent_t e = g_event_pool.back();
    g_event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

class LaunchScope {
 public:
  LaunchScope(int kind, cudaStream_t s, double flops, double bytes) : s_(s) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    std::lock_guard<std::mutex> lock(g_prof_mu);
    if (!g_prof_on) return;
    rec_.kind = kind;
    rec_.flops = flops;
    rec_.bytes = bytes;
    rec_.start = pooled_event();
    rec_.stop = pooled_event();
    active_ = rec_.start && rec_.stop && cudaEventRecord(rec_.start, s_) == cudaSuccess;
  }
  ~LaunchScope() {
    if (!active_) return;
    if (cudaEventRecord(rec_.stop, s_) != cudaSuccess) return;
    std::lock_guard<std::mutex> lock(g_prof_mu);
    g_prof.push_back(rec_);
  }

 private:
  cudaStream_t s_;
  ProfRecord rec_{};
  bool active_ = false;
};

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(PS_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

struct DeviceState {
  bool ready = false;
  int sms = 0;
  int* status = nullptr;  // device address of ps::g_status on this device
  bool smem_attr[kNumVariants] = {};
  bool pair_ready[kNumVariants] = {};
  int pair_clusters[kNumVariants] = {};
  bool chain_ready = false;
  int chain_clusters = 0;
  bool circ_ready = false;
  int circ_clusters = 0;
  int norm_fused_grid[4] = {};  // resident CTAs of the fused normalisation, by dtype
};

std::mutex g_mu;
DeviceState g_dev[kMaxDevices];

// Per-device set-up, done with that device current: SM count, capability
// check and the device address of the status word.
int device_state(DeviceState** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(PS_ERR_UNSUPPORTED, "device index %d", dev);
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceState& st = g_dev[dev];
  if (!st.ready) {
    int major = 0, minor = 0;
    if ((e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute");
    if ((e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute");
    if (major != 10 || minor != 0)
      return fail(PS_ERR_UNSUPPORTED,
                  "polar_switch_b200 kernels are built for sm_100a (B200); device %d is sm_%d%d",
                  dev, major, minor);
    if ((e = cudaDeviceGetAttribute(&st.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute");
    void* p = nullptr;
    if ((e = cudaGetSymbolAddress(&p, ps::g_status)) != cudaSuccess)
      return cuda_fail(e, "cudaGetSymbolAddress(status)");
    st.status = static_cast<int*>(p);
    st.ready = true;
  }
  *out = &st;
  return PS_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int elem_bytes(int dtype) {
  switch (dtype) {
    case PS_F16:
    case PS_BF16:
      return 2;
    case PS_F32:
      return 4;
    case PS_F64:
      return 8;
    default:
      return 0;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 3-D tiled tensor map over (cols, rows, L) of a row-major batched matrix.
int make_map(CUtensorMap* map, const void* ptr, int dtype, int64_t cols, int64_t rows, int64_t L,
             int64_t ld, int64_t bs, uint32_t box_cols, uint32_t box_rows,
             CUtensorMapSwizzle swizzle) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return fail(PS_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const int eb = elem_bytes(dtype);
  CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if (dtype == PS_F32) dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  if (dtype == PS_BF16) dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(L)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * eb), static_cast<cuuint64_t>(bs * eb)};
  cuuint32_t box[3] = {box_cols, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(PS_ERR_INVALID,
                "cuTensorMapEncodeTiled failed (%d): cols=%lld rows=%lld L=%lld ld=%lld bs=%lld",
                static_cast<int>(r), (long long)cols, (long long)rows, (long long)L,
                (long long)ld, (long long)bs);
  return PS_OK;
}

// Operand maps: K-major tiles are (64 K) x (rows), MN-major tiles are boxes of
// (64 M/N) x (64 K); both with 128-byte swizzle.
int map_kmajor(CUtensorMap* m, const void* p, int64_t k, int64_t mn, int64_t L, int64_t ld,
               int64_t bs, uint32_t rows_box) {
  return make_map(m, p, PS_F16, k, mn, L, ld, bs, 64, rows_box, CU_TENSOR_MAP_SWIZZLE_128B);
}
int map_mnmajor(CUtensorMap* m, const void* p, int64_t mn, int64_t k, int64_t L, int64_t ld,
                int64_t bs) {
  return make_map(m, p, PS_F16, mn, k, L, ld, bs, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B);
}
// Operand map for the CTA-pair kernel: with `inner` (the contiguous extent:
// K for a K-major operand, M/N for an MN-major one) a multiple of 64, a 4-D
// "chunked" view (64 | outer | inner / 64 | L) whose (64, 128, 2, 1) box is a
// whole 128-wide K stage in one TMA (*chunked = 1); otherwise the 3-D map of
// map_kmajor / map_mnmajor (*chunked = 0).
int map_pair_operand(CUtensorMap* m, const void* p, bool mn_major, int64_t inner, int64_t outer,
                     int64_t L, int64_t ld, int64_t bs, int* chunked) {
  if (inner % 64 == 0) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
    if (!enc) return fail(PS_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(outer), static_cast<cuuint64_t>(inner / 64),
                          static_cast<cuuint64_t>(L)};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(ld * 2), 128, static_cast<cuuint64_t>(bs * 2)};
    cuuint32_t box[4] = {64, 128, 2, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(p), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r == CUDA_SUCCESS) {
      *chunked = 1;
      return PS_OK;
    }
  }
  *chunked = 0;
  return mn_major ? map_mnmajor(m, p, inner, outer, L, ld, bs)
                  : map_kmajor(m, p, inner, outer, L, ld, bs, ps::pair::BM);
}

// Output map: 32 x 32 sub-tiles, swizzle matching the epilogue's staging.
int map_out(CUtensorMap* m, const void* p, int dtype, int64_t cols, int64_t rows, int64_t L,
            int64_t ld, int64_t bs) {
  const CUtensorMapSwizzle sw =
      elem_bytes(dtype) == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  return make_map(m, p, dtype, cols, rows, L, ld, bs, 32, 32, sw);
}

// Rows of the B-operand box a K-major B tile needs in the selected kernel.
// Whether a product of this kind on n x n buffers runs on CTA pairs.
bool use_pair(bool square, int64_t n) {
  return g_pair_mode == 1 || (g_pair_mode == 2 && square && n <= kPairMaxN);
}
uint32_t b_box_rows(bool pair) { return pair ? ps::pair::BNH : ps::BN; }

// Same problem as `g`, tiled for the CTA-pair kernel.
ps::pair::PairArgs to_pair(const ps::GemmArgs& g, bool sym) {
  ps::pair::PairArgs a;
  std::memset(&a, 0, sizeof(a));
  a.M = g.M;
  a.N = g.N;
  a.K = g.K;
  a.L = g.L;
  a.alpha = g.alpha;
  a.beta = g.beta;
  a.diag = g.diag;
  a.C = g.C;
  a.c_ld = g.c_ld;
  a.c_bs = g.c_bs;
  a.has_addend = g.has_addend;
  a.has_diag = g.has_diag;
  a.a_tri = g.a_tri;
  a.b_tri = g.b_tri;
  a.store_mirror = g.store_mirror;
  a.same_ab = g.same_ab;
  a.upd = g.upd;
  a.p_dtype = g.p_dtype;
  a.P = g.P;
  a.p_ld = g.p_ld;
  a.p_bs = g.p_bs;
  a.decay = g.decay;
  a.upd_alpha = g.upd_alpha;
  a.a_chunk = g.a_chunk;
  a.b_chunk = g.b_chunk;
  a.a2_chunk = g.a2_chunk;
  a.b2_chunk = g.b2_chunk;
  if (sym) {
    a.tb = (g.M + ps::pair::BM - 1) / ps::pair::BM;
    const int P = (a.tb + 1) / 2;
    a.tiles_per_mat = P * (P + 1) / 2;
  } else {
    a.tiles_m2 = (g.M + 2 * ps::pair::BM - 1) / (2 * ps::pair::BM);
    a.tiles_n = (g.N + ps::pair::BN - 1) / ps::pair::BN;
    a.group_m = a.tiles_m2 < 8 ? a.tiles_m2 : 8;
    a.tiles_per_mat = a.tiles_m2 * a.tiles_n;
  }
  a.total_tiles = a.L * a.tiles_per_mat;
  return a;
}

template <bool A_MN, bool B_MN, bool SYM, int OUT>
int launch_gemm_pair(int variant, const CUtensorMap& ta, const CUtensorMap& ta2,
                     const CUtensorMap& tb, const CUtensorMap& tb2, const CUtensorMap& td,
                     ps::pair::PairArgs args, cudaStream_t stream, DeviceState* st, int kind,
                     double flops, double bytes) {
  auto kern = ps::pair::ps_gemm_pair_kernel<A_MN, B_MN, SYM, OUT>;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(ps::pair::NUM_THREADS);
  cfg.dynamicSmemBytes = ps::pair::SMEM_TOTAL;
  cfg.stream = stream;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  if (!st->pair_ready[variant]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         ps::pair::SMEM_TOTAL);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(pair gemm smem)");
    cfg.gridDim = dim3(2 * (st->sms / 2));
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters");
    if (clusters < 1) return fail(PS_ERR_UNSUPPORTED, "no co-resident CTA pair fits on the device");
    st->pair_clusters[variant] = clusters;
    st->pair_ready[variant] = true;
  }
  if (args.total_tiles <= 0) return PS_OK;
  args.status = st->status;
  args.wait_limit = g_wait_limit;
  int pairs = args.total_tiles < st->pair_clusters[variant] ? args.total_tiles
                                                            : st->pair_clusters[variant];
  if (g_max_ctas > 1 && pairs > g_max_ctas / 2) pairs = g_max_ctas / 2;
  cfg.gridDim = dim3(2 * pairs);
  LaunchScope scope(kind, stream, flops, bytes);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ta, ta2, tb, tb2, td, args);
  if (e != cudaSuccess) return cuda_fail(e, "pair gemm launch");
  return PS_OK;
}

// A GEMM prepared but not yet launched: its maps and arguments, its profiling
// figures, and the launcher of its kernel variant. Jobs of one variant and
// profiling kind can share a launch (ps::GemmBatch).
struct GemmJob;
using JobLauncher = int (*)(const GemmJob* jobs, int n, cudaStream_t stream);
struct GemmJob {
  ps::GemmProblem prob;
  JobLauncher launch;
  int variant, kind;
  bool pair;  // run on the CTA-pair kernel
  double flops, bytes;
};

// While a sink is installed on this thread, launch_gemm collects jobs instead
// of launching them; flush_jobs then launches them batched.
thread_local std::vector<GemmJob>* g_job_sink = nullptr;

template <bool A_MN, bool B_MN, bool SYM, int OUT>
int launch_jobs(const GemmJob* jobs, int n, cudaStream_t stream) {
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  const int variant = jobs[0].variant;
  if (jobs[0].pair) {
    for (int i = 0; i < n; ++i) {
      const ps::GemmProblem& q = jobs[i].prob;
      if ((rc = launch_gemm_pair<A_MN, B_MN, SYM, OUT>(variant, q.tmA, q.tmA2, q.tmB, q.tmB2, q.tmD,
                                                        to_pair(q.args, SYM), stream, st,
                                                        jobs[i].kind, jobs[i].flops, jobs[i].bytes)))
        return rc;
    }
    return PS_OK;
  }
  auto kern1 = ps::ps_gemm_kernel<A_MN, B_MN, SYM, OUT, false>;
  auto kernb = ps::ps_gemm_kernel<A_MN, B_MN, SYM, OUT, true>;
  if (!st->smem_attr[variant]) {
    cudaError_t e =
        cudaFuncSetAttribute(kern1, cudaFuncAttributeMaxDynamicSharedMemorySize, ps::SMEM_TOTAL);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(kernb, cudaFuncAttributeMaxDynamicSharedMemorySize, ps::SMEM_TOTAL);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm smem)");
    st->smem_attr[variant] = true;
  }
  for (int i0 = 0; i0 < n; i0 += ps::MAX_BATCH) {
    const int cnt = n - i0 < ps::MAX_BATCH ? n - i0 : ps::MAX_BATCH;
    ps::GemmBatch batch;
    std::memset(&batch, 0, sizeof(batch));
    double flops = 0.0, bytes = 0.0;
    int total = 0, used = 0;
    for (int i = 0; i < cnt; ++i) {
      const GemmJob& j = jobs[i0 + i];
      if (j.prob.args.total_tiles <= 0) continue;
      batch.p[used] = j.prob;
      batch.p[used].args.status = st->status;
      batch.p[used].args.wait_limit = g_wait_limit;
      batch.tile_start[used] = total;
      total += j.prob.args.total_tiles;
      flops += j.flops;
      bytes += j.bytes;
      ++used;
    }
    if (used == 0) continue;
    batch.count = used;
    batch.tile_start[used] = total;
    int grid = total < st->sms ? total : st->sms;
    if (g_max_ctas > 0 && grid > g_max_ctas) grid = g_max_ctas;
    LaunchScope scope(jobs[i0].kind, stream, flops, bytes);
    if (used == 1)
      kern1<<<grid, ps::NUM_THREADS, ps::SMEM_TOTAL, stream>>>(batch);
    else
      kernb<<<grid, ps::NUM_THREADS, ps::SMEM_TOTAL, stream>>>(batch);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
  }
  return PS_OK;
}

// Launches collected jobs: jobs of one variant and kind share launches (they
// are independent, so their order does not matter).
int flush_jobs(std::vector<GemmJob>& jobs, cudaStream_t stream) {
  std::vector<bool> done(jobs.size(), false);
  std::vector<GemmJob> group;
  for (size_t i = 0; i < jobs.size(); ++i) {
    if (done[i]) continue;
    group.clear();
    for (size_t k = i; k < jobs.size(); ++k) {
      if (!done[k] && jobs[k].launch == jobs[i].launch && jobs[k].kind == jobs[i].kind &&
          jobs[k].pair == jobs[i].pair) {
        group.push_back(jobs[k]);
        done[k] = true;
      }
    }
    const int rc = jobs[i].launch(group.data(), static_cast<int>(group.size()), stream);
    if (rc) return rc;
  }
  jobs.clear();
  return PS_OK;
}

// Installs a job sink for the current scope (see g_job_sink).
struct JobSink {
  std::vector<GemmJob> jobs;
  std::vector<GemmJob>* prev;
  JobSink() : prev(g_job_sink) { g_job_sink = &jobs; }
  ~JobSink() { g_job_sink = prev; }
  int flush(cudaStream_t s) {
    g_job_sink = prev;
    return flush_jobs(jobs, s);
  }
};

// ta2 / tb2: the operands' maps in the other majorness, read only when the
// operand is triangle-stored (args.a_tri / b_tri).
template <bool A_MN, bool B_MN, bool SYM, int OUT>
int launch_gemm(int variant, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td,
                ps::GemmArgs args, cudaStream_t stream, int kind, double flops, double bytes,
                bool pair, const CUtensorMap* ta2 = nullptr, const CUtensorMap* tb2 = nullptr) {
  if ((args.a_tri && !ta2) || (args.b_tri && !tb2))
    return fail(PS_ERR_INVALID, "internal: triangle-stored operand without its second map");
  GemmJob job;
  std::memset(&job, 0, sizeof(job));
  job.prob.tmA = ta;
  job.prob.tmA2 = ta2 ? *ta2 : ta;
  job.prob.tmB = tb;
  job.prob.tmB2 = tb2 ? *tb2 : tb;
  job.prob.tmD = td;
  job.prob.args = args;
  job.launch = &launch_jobs<A_MN, B_MN, SYM, OUT>;
  job.variant = variant;
  job.kind = kind;
  job.pair = pair;
  job.flops = flops;
  job.bytes = bytes;
  if (g_job_sink) {
    g_job_sink->push_back(job);
    return PS_OK;
  }
  return launch_jobs<A_MN, B_MN, SYM, OUT>(&job, 1, stream);
}

// ------------------------------------------------------------------ chain
// Whether the inner iterations of an n-group run as chain launches.
bool use_chain(int64_t n, int buffers) {
  return g_chain_mode && use_pair(true, n) && buffers <= ps::chain::MAX_BUFS;
}

// Pair tiles of one n x n symmetric product (column pair p owns row pairs 0..p).
int pair_sym_tiles(int64_t n) {
  const int tb = static_cast<int>((n + ps::pair::BM - 1) / ps::pair::BM);
  const int P = (tb + 1) / 2;
  return P * (P + 1) / 2;
}

// Inner iterations steps[0..S) (S <= MAX_STEPS) of L triangle-stored n x n
// buffers (buffer k at bufs + k * buf_bytes) as one chain launch. `done`
// holds L counters whose value at the launch is `base`; every pair tile adds
// SIGNALS_PER_TILE to its matrix's counter.
int chain_launch(uint8_t* bufs, int64_t buf_bytes, int buffers, int64_t L, int64_t n,
                 const ps_step* steps, int S, unsigned* done, unsigned base, cudaStream_t stream,
                 long long dep_limit = 0) {
  using ps::chain::ChainParams;
  if (S < 1 || S > ps::chain::MAX_STEPS || buffers > ps::chain::MAX_BUFS)
    return fail(PS_ERR_INVALID, "internal: chain of %d steps over %d buffers", S, buffers);
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  auto kern = ps::chain::ps_chain_pair_kernel;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(ps::pair::NUM_THREADS);
  cfg.dynamicSmemBytes = ps::pair::SMEM_TOTAL;
  cfg.stream = stream;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  if (!st->chain_ready) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         ps::pair::SMEM_TOTAL);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(chain smem)");
    cfg.gridDim = dim3(2 * (st->sms / 2));
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters(chain)");
    if (clusters < 1) return fail(PS_ERR_UNSUPPORTED, "no co-resident CTA pair fits on the device");
    st->chain_clusters = clusters;
    st->chain_ready = true;
  }
  // Params are large (~6 KB); kept off the stack.
  static thread_local ChainParams P;
  std::memset(&P, 0, sizeof(P));
  int ck = 1, cm = 1;
  for (int k = 0; k < buffers; ++k) {
    void* ptr = bufs + k * buf_bytes;
    int c1 = 0, c2 = 0;
    if ((rc = map_pair_operand(&P.tmK[k], ptr, false, n, n, L, n, n * n, &c1))) return rc;
    if ((rc = map_pair_operand(&P.tmMN[k], ptr, true, n, n, L, n, n * n, &c2))) return rc;
    if ((rc = map_out(&P.tmD[k], ptr, PS_F16, n, n, L, n, n * n))) return rc;
    P.buf[k] = static_cast<const __half*>(ptr);
    ck &= c1;
    cm &= c2;
  }
  if (ck != cm) return fail(PS_ERR_INVALID, "internal: chain operand maps disagree on the chunked layout");
  P.chunked = ck;
  for (int i = 0; i < S; ++i)
    P.steps[i] = {steps[i].dst, steps[i].src, steps[i].add, steps[i].alpha, steps[i].beta,
                  steps[i].diag};
  const int T = pair_sym_tiles(n);
  int pairs = st->chain_clusters;
  if (g_max_ctas > 1 && pairs > g_max_ctas / 2) pairs = g_max_ctas / 2;
  // Chunk size: the tile a producer waits for (step s - 1 of its matrix) was
  // scheduled S chunks earlier; make that about two waves of pair tiles, and
  // keep the item table within MAX_ITEMS.
  int64_t C = (2LL * pairs + static_cast<int64_t>(S) * T - 1) / (static_cast<int64_t>(S) * T);
  if (C < 1) C = 1;
  const int64_t c_min = (L * S + ps::chain::MAX_ITEMS - 1) / ps::chain::MAX_ITEMS;
  if (C < c_min) C = c_min;
  if (C > L) C = L;
  const int64_t nch = (L + C - 1) / C;
  int items = 0;
  int64_t tiles = 0;
  for (int64_t round = 0; round < nch + S - 1; ++round) {
    for (int s = 0; s < S; ++s) {
      const int64_t c = round - s;
      if (c < 0 || c >= nch) continue;
      P.item_start[items] = static_cast<int>(tiles);
      P.item_step[items] = static_cast<unsigned short>(s);
      P.item_chunk[items] = static_cast<unsigned short>(c);
      ++items;
      const int64_t size = std::min<int64_t>(C, L - c * C);
      tiles += size * T;
    }
  }
  if (tiles > INT32_MAX) return fail(PS_ERR_UNSUPPORTED, "chain: too many tiles");
  P.item_start[items] = static_cast<int>(tiles);
  P.n_items = items;
  P.total_tiles = static_cast<int>(tiles);
  P.n = static_cast<int>(n);
  P.L = static_cast<int>(L);
  P.T = T;
  P.chunk = static_cast<int>(C);
  P.nbufs = buffers;
  P.base = base;
  P.done = done;
  P.status = st->status;
  P.wait_limit = g_wait_limit;
  P.dep_limit = dep_limit > 0 ? dep_limit : g_wait_limit;
  if (pairs > P.total_tiles) pairs = P.total_tiles;
  cfg.gridDim = dim3(2 * pairs);
  const double nn = static_cast<double>(n) * n;
  LaunchScope scope(kProfSquare, stream, static_cast<double>(S) * L * nn * n,
                    static_cast<double>(S) * L * nn * 2.0 * 3.0);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, P);
  if (e != cudaSuccess) return cuda_fail(e, "chain launch");
  return PS_OK;
}

void fill_sym_tiles(ps::GemmArgs& a, int64_t n, int64_t L) {
  a.tb = static_cast<int>((n + ps::BM - 1) / ps::BM);
  int per = 0;
  for (int bi = 0; bi < a.tb; ++bi) per += (a.tb - bi + 1) / 2;
  a.tiles_per_mat = per;
  a.total_tiles = static_cast<int>(L * per);
  a.tiles_m = a.tiles_n = 0;
  a.group_m = 1;
}

void fill_gen_tiles(ps::GemmArgs& a, int64_t M, int64_t N, int64_t L) {
  a.tiles_m = static_cast<int>((M + ps::BM - 1) / ps::BM);
  a.tiles_n = static_cast<int>((N + ps::BN - 1) / ps::BN);
  a.group_m = a.tiles_m < 16 ? a.tiles_m : 16;
  a.tiles_per_mat = a.tiles_m * a.tiles_n;
  a.total_tiles = static_cast<int>(L * a.tiles_per_mat);
  a.tb = 0;
}

ps::GemmArgs base_args(int64_t M, int64_t N, int64_t K, int64_t L) {
  ps::GemmArgs a;
  std::memset(&a, 0, sizeof(a));
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.L = static_cast<int>(L);
  a.alpha = 1.f;
  a.store_mirror = 1;
  return a;
}

bool dims_ok(int64_t L, int64_t r, int64_t c) {
  const int64_t lim = int64_t(1) << 30;
  return L > 0 && r > 0 && c > 0 && L < lim && r < lim && c < lim && L * r * c < (int64_t(1) << 46);
}

// ------------------------------------------------------------------ ops
int sym_product_impl(const void* p, const void* q, const void* c, void* out, int64_t L,
                     int64_t n, float alpha, float beta, float diag, cudaStream_t stream,
                     const char* name, bool tri = false) {
  if (!p || !q || !out) return fail(PS_ERR_INVALID, "%s: null pointer", name);
  if (!dims_ok(L, n, n)) return fail(PS_ERR_INVALID, "%s: bad sizes", name);
  if (n % 8) return fail(PS_ERR_INVALID, "%s: n=%lld must be a multiple of 8", name, (long long)n);
  if (!aligned16(p) || !aligned16(q) || !aligned16(out) || (c && !aligned16(c)))
    return fail(PS_ERR_INVALID, "%s: pointers must be 16-byte aligned", name);
  if (out == p || out == q)
    return fail(PS_ERR_INVALID, "%s: the output must not be a multiplied operand", name);
  CUtensorMap ta, tb, td;
  int rc;
  // A squared buffer is read as A . A^T (both operands K-major, the reference
  // Triton kernel's form); a product of two different matrices is A @ B with B
  // read MN-major from its row-major storage, exactly the reference's
  // gemm_symmetric(A, B) even when B is symmetric only up to rounding.
  const bool same = p == q;
  const bool pair = use_pair(same, n);
  ps::GemmArgs a = base_args(n, n, n, L);
  if (pair) {
    if ((rc = map_pair_operand(&ta, p, false, n, n, L, n, n * n, &a.a_chunk))) return rc;
    if ((rc = map_pair_operand(&tb, q, !same, n, n, L, n, n * n, &a.b_chunk))) return rc;
  } else {
    if ((rc = map_kmajor(&ta, p, n, n, L, n, n * n, ps::BM))) return rc;
    if (same) {
      if ((rc = map_kmajor(&tb, q, n, n, L, n, n * n, b_box_rows(pair)))) return rc;
    } else {
      if ((rc = map_mnmajor(&tb, q, n, n, L, n, n * n))) return rc;
    }
  }
  if ((rc = map_out(&td, out, PS_F16, n, n, L, n, n * n))) return rc;
  fill_sym_tiles(a, n, L);
  a.alpha = alpha;
  a.beta = beta;
  a.diag = diag;
  a.C = static_cast<const __half*>(c);
  a.c_ld = n;
  a.c_bs = n * n;
  a.has_addend = c != nullptr;
  a.has_diag = diag != 0.f;
  a.same_ab = same ? 1 : 0;  // ta and tb above: same pointer, shape and box
  const double nn = static_cast<double>(n) * n;
  const double bytes = L * nn * 2.0 * ((same ? 1 : 2) + (c ? 1 : 0) + 1);
  if (same && tri) {
    // squared operand and result both held as upper-triangle blocks
    CUtensorMap tm;
    if (pair) {
      if ((rc = map_pair_operand(&tm, p, true, n, n, L, n, n * n, &a.a2_chunk))) return rc;
      a.b2_chunk = a.a2_chunk;
    } else if ((rc = map_mnmajor(&tm, p, n, n, L, n, n * n))) {
      return rc;
    }
    a.a_tri = a.b_tri = 1;
    a.store_mirror = 0;
    return launch_gemm<false, false, true, ps::kOutF16>(0, ta, tb, td, a, stream, kProfSquare,
                                                        L * nn * n, bytes, pair, &tm, &tm);
  }
  if (same)
    return launch_gemm<false, false, true, ps::kOutF16>(0, ta, tb, td, a, stream, kProfSquare,
                                                        L * nn * n, bytes, pair);
  return launch_gemm<false, true, true, ps::kOutF16>(8, ta, tb, td, a, stream, kProfSquare,
                                                     L * nn * n, bytes, pair);
}

int gram_impl(const void* x, void* out, int64_t L, int64_t rows, int64_t cols, int64_t x_ld,
              bool tall, cudaStream_t stream, bool tri_out = false) {
  if (!x || !out) return fail(PS_ERR_INVALID, "ps_gram: null pointer");
  if (!dims_ok(L, rows, cols) || x_ld < cols)
    return fail(PS_ERR_INVALID, "ps_gram: bad sizes");
  if (x_ld % 8) return fail(PS_ERR_INVALID, "ps_gram: x_ld must be a multiple of 8");
  if (!aligned16(x) || !aligned16(out))
    return fail(PS_ERR_INVALID, "ps_gram: pointers must be 16-byte aligned");
  const int64_t n = tall ? cols : rows, K = tall ? rows : cols;
  if (n % 8) return fail(PS_ERR_INVALID, "ps_gram: min(rows, cols) must be a multiple of 8");
  CUtensorMap ta, tb, td;
  int rc;
  if ((rc = map_out(&td, out, PS_F16, n, n, L, n, n * n))) return rc;
  ps::GemmArgs a = base_args(n, n, K, L);
  fill_sym_tiles(a, n, L);
  a.store_mirror = tri_out ? 0 : 1;
  const double flops = static_cast<double>(L) * n * n * K;
  const double bytes = static_cast<double>(L) * 2.0 * (static_cast<double>(n) * K + n * n);
  const bool pair = use_pair(false, n);
  // both operands read through one map: diagonal pair tiles stage their rows once
  a.same_ab = pair ? 1 : 0;
  if (!tall) {
    if (pair) {
      if ((rc = map_pair_operand(&ta, x, false, K, n, L, x_ld, rows * x_ld, &a.a_chunk))) return rc;
      tb = ta;
      a.b_chunk = a.a_chunk;
    } else {
      if ((rc = map_kmajor(&ta, x, K, n, L, x_ld, rows * x_ld, ps::BM))) return rc;
      if ((rc = map_kmajor(&tb, x, K, n, L, x_ld, rows * x_ld, b_box_rows(pair)))) return rc;
    }
    return launch_gemm<false, false, true, ps::kOutF16>(0, ta, tb, td, a, stream, kProfGram,
                                                        flops, bytes, pair);
  }
  if (pair) {
    if ((rc = map_pair_operand(&ta, x, true, n, K, L, x_ld, rows * x_ld, &a.a_chunk))) return rc;
    a.b_chunk = a.a_chunk;
  } else if ((rc = map_mnmajor(&ta, x, n, K, L, x_ld, rows * x_ld))) {
    return rc;
  }
  return launch_gemm<true, true, true, ps::kOutF16>(1, ta, ta, td, a, stream, kProfGram, flops,
                                                    bytes, pair);
}

template <int OUT>
int apply_launch(bool tall, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td,
                 const ps::GemmArgs& a, cudaStream_t s, const CUtensorMap* t2, bool pair) {
  const double M = a.M, N = a.N, K = a.K, L = a.L;
  const double out_bytes = OUT == ps::kOutF32 ? 4.0 : 2.0;
  const double flops = 2.0 * L * M * N * K;
  const double bytes = L * (2.0 * K * K + 2.0 * M * N + out_bytes * M * N);
  (void)tall;  // both orientations are A (K-major) times B (MN-major)
  return launch_gemm<false, true, false, OUT>(2 + OUT, ta, tb, td, a, s, kProfApply, flops, bytes,
                                              pair, a.a_tri ? t2 : nullptr, a.b_tri ? t2 : nullptr);
}

int apply_impl(const void* b, const void* x, void* y, int64_t L, int64_t rows, int64_t cols,
               int64_t x_ld, float residual, int y_dtype, int64_t y_ld, bool tall,
               cudaStream_t stream, bool tri_b = false, const ps_update* upd = nullptr) {
  if (upd && upd->p) {
    // Muon update into a parameter bank instead of storing y (CTA-pair path;
    // the caller has checked the layout): y only needs to be a valid
    // description of the (L, rows, cols) output for the maps.
    if (!use_pair(false, tall ? cols : rows))
      return fail(PS_ERR_UNSUPPORTED, "update-fused apply needs the CTA-pair kernel");
  }
  if (!b || !x || !y) return fail(PS_ERR_INVALID, "ps_apply: null pointer");
  if (!dims_ok(L, rows, cols) || x_ld < cols || y_ld < cols)
    return fail(PS_ERR_INVALID, "ps_apply: bad sizes");
  if (y_dtype != PS_F16 && y_dtype != PS_F32 && y_dtype != PS_BF16)
    return fail(PS_ERR_INVALID, "ps_apply: y_dtype must be PS_F16, PS_F32 or PS_BF16");
  if (x_ld % 8 || (y_ld * elem_bytes(y_dtype)) % 16)
    return fail(PS_ERR_INVALID, "ps_apply: row pitches must be multiples of 16 bytes");
  if (!aligned16(b) || !aligned16(x) || !aligned16(y))
    return fail(PS_ERR_INVALID, "ps_apply: pointers must be 16-byte aligned");
  if (y == x || y == b) return fail(PS_ERR_INVALID, "ps_apply: y must not alias x or b");
  const int64_t n = tall ? cols : rows, m = tall ? rows : cols;
  if (n % 8) return fail(PS_ERR_INVALID, "ps_apply: min(rows, cols) must be a multiple of 8");
  CUtensorMap ta, tb, td;
  int rc;
  const int64_t M = tall ? m : n, N = tall ? n : m;
  const bool pair = use_pair(false, n);
  ps::GemmArgs a = base_args(M, N, n, L);
  if ((rc = map_out(&td, y, y_dtype, N, M, L, y_ld, rows * y_ld))) return rc;
  if (pair) {
    if (!tall) {
      if ((rc = map_pair_operand(&ta, b, false, n, n, L, n, n * n, &a.a_chunk))) return rc;
      if ((rc = map_pair_operand(&tb, x, true, m, n, L, x_ld, rows * x_ld, &a.b_chunk))) return rc;
    } else {
      if ((rc = map_pair_operand(&ta, x, false, n, m, L, x_ld, rows * x_ld, &a.a_chunk))) return rc;
      if ((rc = map_pair_operand(&tb, b, true, n, n, L, n, n * n, &a.b_chunk))) return rc;
    }
  } else if (!tall) {
    if ((rc = map_kmajor(&ta, b, n, n, L, n, n * n, ps::BM))) return rc;
    if ((rc = map_mnmajor(&tb, x, m, n, L, x_ld, rows * x_ld))) return rc;
  } else {
    // X @ B: B read MN-major (row-major B, element (k, n)), exactly X @ B.
    if ((rc = map_kmajor(&ta, x, n, m, L, x_ld, rows * x_ld, ps::BM))) return rc;
    if ((rc = map_mnmajor(&tb, b, n, n, L, n, n * n))) return rc;
  }
  fill_gen_tiles(a, M, N, L);
  if (upd && upd->p) {
    a.upd = 1;
    a.p_dtype = upd->p_dtype == PS_F32 ? ps::kOutF32 : upd->p_dtype == PS_BF16 ? ps::kOutBF16
                                                                               : ps::kOutF16;
    a.P = upd->p;
    a.p_ld = cols;
    a.p_bs = rows * cols;
    a.decay = upd->decay;
    a.upd_alpha = upd->alpha;
  }
  if (residual != 0.f) {
    a.has_addend = 1;
    a.beta = residual;
    a.C = static_cast<const __half*>(x);
    a.c_ld = x_ld;
    a.c_bs = rows * x_ld;
  }
  // b held as upper-triangle blocks: its second map has the other majorness
  CUtensorMap t2;
  if (tri_b) {
    if (!tall) {
      if (pair) {
        if ((rc = map_pair_operand(&t2, b, true, n, n, L, n, n * n, &a.a2_chunk))) return rc;
      } else if ((rc = map_mnmajor(&t2, b, n, n, L, n, n * n))) {
        return rc;
      }
      a.a_tri = 1;
    } else {
      if (pair) {
        if ((rc = map_pair_operand(&t2, b, false, n, n, L, n, n * n, &a.b2_chunk))) return rc;
      } else if ((rc = map_kmajor(&t2, b, n, n, L, n, n * n, b_box_rows(false)))) {
        return rc;
      }
      a.b_tri = 1;
    }
  }
  switch (y_dtype) {
    case PS_F16:
      return apply_launch<ps::kOutF16>(tall, ta, tb, td, a, stream, &t2, pair);
    case PS_F32:
      return apply_launch<ps::kOutF32>(tall, ta, tb, td, a, stream, &t2, pair);
    default:
      return apply_launch<ps::kOutBF16>(tall, ta, tb, td, a, stream, &t2, pair);
  }
}

int add_diag_impl(const void* in, void* out, int64_t L, int64_t n, float a, cudaStream_t stream) {
  if (!in || !out) return fail(PS_ERR_INVALID, "ps_add_diag: null pointer");
  if (!dims_ok(L, n, n)) return fail(PS_ERR_INVALID, "ps_add_diag: bad sizes");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  int64_t blocks = (L * n * n + ps::NORM_THREADS - 1) / ps::NORM_THREADS;
  if (blocks > 8LL * st->sms) blocks = 8LL * st->sms;
  LaunchScope scope(kProfOther, stream, 0.0, 4.0 * L * n * n);
  ps::ps_add_diag_kernel<<<static_cast<unsigned>(blocks), ps::NORM_THREADS, 0, stream>>>(
      static_cast<const __half*>(in), static_cast<__half*>(out), L, n, a);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PS_OK : cuda_fail(e, "add_diag launch");
}

// ------------------------------------------------------------------ normalise
int norm_chunks(int64_t L, int64_t rows, int64_t cols, int sms) {
  // Enough blocks in flight for HBM bandwidth: about 4 per SM in total.
  const int64_t E = rows * cols;
  int64_t want = (4LL * sms + L - 1) / L;
  const int64_t max_by_size = (E + 4095) / 4096;  // at least 4096 elements per block
  if (want > max_by_size) want = max_by_size;
  if (want > rows) want = rows;  // strided path splits by rows
  if (want < 1) want = 1;
  if (want > 1024) want = 1024;
  return static_cast<int>(want);
}

int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// Canonical chunk count of a contiguous matrix of E elements (ps_norm.cuh).
int64_t norm_flat_chunks(int64_t E) {
  const int64_t ce = ps::norm_chunk_elems(E);
  return (E + ce - 1) / ce;
}

// Partial sums one matrix may need: canonical chunks (contiguous input) or
// row ranges (strided input).
int64_t norm_partials_per_matrix(int64_t L, int64_t rows, int64_t cols, int sms) {
  const int64_t a = norm_flat_chunks(rows * cols), b = norm_chunks(L, rows, cols, sms);
  return a > b ? a : b;
}

// Largest grid y extent; launches that put matrices on grid y cover longer
// batches in slices of this many matrices.
constexpr int64_t kMaxGridY = 65535;

// Pass 1: chunk sums of squares. Contiguous input is summed over chunks of
// `chunk_elems` elements, strided input over `chunks` row ranges; returns the
// number of chunk sums per matrix through `chunks_out`.
template <typename T>
int launch_norm_pass1(const void* x, int64_t L, int64_t R, int64_t C, int64_t sL, int64_t sR,
                      int64_t sC, double* partial, int chunks, int64_t chunk_elems, int* chunks_out,
                      cudaStream_t s) {
  const int flat = (sC == 1 && sR == C) ? 1 : 0;
  if (flat) chunks = static_cast<int>((R * C + chunk_elems - 1) / chunk_elems);
  *chunks_out = chunks;
  for (int64_t l0 = 0; l0 < L; l0 += kMaxGridY) {  // matrices run along grid y
    const int64_t n = L - l0 < kMaxGridY ? L - l0 : kMaxGridY;
    dim3 g1(chunks, static_cast<unsigned>(n));
    LaunchScope scope(kProfNormalize, s, 2.0 * n * R * C, static_cast<double>(n) * R * C * sizeof(T));
    ps::ps_norm_partial_kernel<T><<<g1, ps::NORM_THREADS, 0, s>>>(
        static_cast<const T*>(x) + l0 * sL, R, C, sL, sR, sC, flat, chunks, chunk_elems,
        partial + l0 * chunks);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "normalize launch (pass 1)");
  }
  return PS_OK;
}

// Pass 2: xh = fp16(x / den) with den from `chunks` sums per matrix (partial
// == nullptr: den = 1, a plain FP16 rounding).
template <typename T>
int launch_norm_pass2(const void* x, int64_t L, int64_t R, int64_t C, int64_t sL, int64_t sR,
                      int64_t sC, const double* partial, int chunks, float eps, void* xh, int64_t Rp,
                      int64_t Cp, int sms, cudaStream_t s) {
  const int flat = (sC == 1 && sR == C) ? 1 : 0;
  const int64_t per_mat_blocks = (Rp * Cp + ps::NORM_THREADS * 8 - 1) / (ps::NORM_THREADS * 8);
  int64_t gx = (4LL * sms + L - 1) / L;
  if (gx > per_mat_blocks) gx = per_mat_blocks;
  if (gx < 1) gx = 1;
  for (int64_t l0 = 0; l0 < L; l0 += kMaxGridY) {  // matrices run along grid y
    const int64_t n = L - l0 < kMaxGridY ? L - l0 : kMaxGridY;
    dim3 g2(static_cast<unsigned>(gx), static_cast<unsigned>(n));
    LaunchScope scope(kProfNormalize, s, static_cast<double>(n) * R * C,
                      static_cast<double>(n) * R * C * sizeof(T) + 2.0 * n * Rp * Cp);
    ps::ps_scale_cast_kernel<T><<<g2, ps::NORM_THREADS, 0, s>>>(
        static_cast<const T*>(x) + l0 * sL, R, C, sL, sR, sC, flat,
        partial ? partial + l0 * chunks : nullptr, chunks, eps,
        static_cast<__half*>(xh) + l0 * Rp * Cp, Rp, Cp);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "normalize launch (pass 2)");
  }
  return PS_OK;
}

// Two passes.
template <typename T>
int launch_normalize(const void* x, int64_t L, int64_t R, int64_t C, int64_t sL, int64_t sR,
                     int64_t sC, float eps, void* xh, int64_t Rp, int64_t Cp, double* partial,
                     int chunks, int64_t chunk_elems, int sms, cudaStream_t s) {
  int nch = 0;
  int rc = launch_norm_pass1<T>(x, L, R, C, sL, sR, sC, partial, chunks, chunk_elems, &nch, s);
  if (rc) return rc;
  return launch_norm_pass2<T>(x, L, R, C, sL, sR, sC, partial, nch, eps, xh, Rp, Cp, sms, s);
}

int64_t normalize_ws_bytes(int64_t L, int64_t rows, int64_t cols, int sms) {
  return round_up(L * norm_partials_per_matrix(L, rows, cols, sms) *
                      static_cast<int64_t>(sizeof(double)),
                  256);
}

int normalize_impl(const void* x, int x_dtype, int64_t L, int64_t rows, int64_t cols, int64_t sL,
                   int64_t sR, int64_t sC, float eps, void* xh, int64_t Rp, int64_t Cp, void* ws,
                   int64_t ws_bytes, cudaStream_t stream) {
  if (!x || !xh || !ws) return fail(PS_ERR_INVALID, "ps_normalize: null pointer");
  if (!dims_ok(L, rows, cols) || Rp < rows || Cp < cols)
    return fail(PS_ERR_INVALID, "ps_normalize: bad sizes");
  if (elem_bytes(x_dtype) == 0) return fail(PS_ERR_INVALID, "ps_normalize: bad dtype");
  if (!(eps > 0.f)) return fail(PS_ERR_INVALID, "ps_normalize: eps must be positive");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  const int chunks = norm_chunks(L, rows, cols, st->sms);
  if (ws_bytes < normalize_ws_bytes(L, rows, cols, st->sms))
    return fail(PS_ERR_WORKSPACE, "ps_normalize: workspace too small");
  double* partial = static_cast<double*>(ws);
  const int64_t ce = ps::norm_chunk_elems(rows * cols);
  switch (x_dtype) {
    case PS_F16:
      return launch_normalize<__half>(x, L, rows, cols, sL, sR, sC, eps, xh, Rp, Cp, partial,
                                      chunks, ce, st->sms, stream);
    case PS_BF16:
      return launch_normalize<__nv_bfloat16>(x, L, rows, cols, sL, sR, sC, eps, xh, Rp, Cp,
                                             partial, chunks, ce, st->sms, stream);
    case PS_F32:
      return launch_normalize<float>(x, L, rows, cols, sL, sR, sC, eps, xh, Rp, Cp, partial,
                                     chunks, ce, st->sms, stream);
    default:
      return launch_normalize<double>(x, L, rows, cols, sL, sR, sC, eps, xh, Rp, Cp, partial,
                                      chunks, ce, st->sms, stream);
  }
}

// One normalisation of a grouped circuit: the arguments of normalize_impl.
struct NormJob {
  const void* x;
  int x_dtype;
  int64_t L, R, C, sL, sR, sC;
  void* xh;
  int64_t Rp, Cp;
  double* partial;
  unsigned* count;  // L zeroed counters for the fused kernel (nullptr: two passes)
};

// Resident CTAs of the fused normalisation for input type T on this device
// (one NORM_CHUNK chunk of T in shared memory per CTA); 0 if it cannot run.
template <typename T>
int norm_fused_grid(DeviceState* st, int dtype) {
  if (st->norm_fused_grid[dtype]) return st->norm_fused_grid[dtype];
  auto kern = ps::ps_normalize_fused_kernel<T>;
  const int smem = ps::NORM_CHUNK * static_cast<int>(sizeof(T));
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, ps::NORM_THREADS, smem) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  st->norm_fused_grid[dtype] = per_sm * st->sms;
  return st->norm_fused_grid[dtype];
}

// Whether a job can take the fused kernel: contiguous, unpadded, aligned, and
// every matrix's chunks (of NORM_CHUNK elements) fit in the resident grid.
bool norm_fused_ok(const NormJob& j, int grid, int elem) {
  const int64_t E = j.R * j.C;
  const int64_t nch = (E + ps::NORM_CHUNK - 1) / ps::NORM_CHUNK;
  return g_norm_fused && j.count && grid > 0 && j.sC == 1 && j.sR == j.C && j.sL == E &&
         j.Rp == j.R && j.Cp == j.C && E % 8 == 0 && (E * elem) % 16 == 0 && aligned16(j.x) &&
         aligned16(j.xh) && nch <= ps::NORM_MAX_CHUNKS && nch <= grid;
}

template <typename T>
int launch_normalize_fused(const NormJob* jobs, int n, float eps, DeviceState* st, int grid,
                           cudaStream_t s) {
  ps::NormFused f;
  std::memset(&f, 0, sizeof(f));
  f.count = n;
  f.eps = eps;
  f.status = st->status;
  f.wait_limit = g_wait_limit;
  long long t = 0;
  double elems = 0.0;
  for (int i = 0; i < n; ++i) {
    const NormJob& j = jobs[i];
    ps::NormFusedProblem& q = f.p[i];
    q.x = j.x;
    q.xh = static_cast<__half*>(j.xh);
    q.partial = j.partial;
    q.count = j.count;
    q.E = j.R * j.C;
    q.chunks = static_cast<int>((q.E + ps::NORM_CHUNK - 1) / ps::NORM_CHUNK);
    q.t0 = t;
    t += j.L * q.chunks;
    elems += static_cast<double>(j.L) * q.E;
  }
  f.total = t;
  const int g = static_cast<int>(t < grid ? t : grid);
  LaunchScope scope(kProfNormalize, s, 3.0 * elems, elems * (sizeof(T) + 2.0));
  ps::ps_normalize_fused_kernel<T>
      <<<g, ps::NORM_THREADS, ps::NORM_CHUNK * sizeof(T), s>>>(f);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PS_OK : cuda_fail(e, "fused normalize launch");
}


// Both passes of up to NORM_BATCH_MAX normalisations with input type T, one
// launch per pass. Each matrix keeps normalize_impl's chunk count and chunk
// size, so its chunk sums, their ordered sum and every FP16 output are the
// same bits as in a launch of its own; only the split of the scale-and-cast
// pass into blocks differs (sized by each problem's share of the elements),
// and no output depends on that split.
template <typename T>
int launch_normalize_batch(const NormJob* jobs, int n, float eps, int sms, cudaStream_t s) {
  ps::NormBatch b1, b2;
  std::memset(&b1, 0, sizeof(b1));
  std::memset(&b2, 0, sizeof(b2));
  b1.count = b2.count = n;
  b1.eps = b2.eps = eps;
  double elems = 0.0, in_bytes = 0.0, out_bytes = 0.0;
  for (int i = 0; i < n; ++i) {
    elems += static_cast<double>(jobs[i].L) * jobs[i].R * jobs[i].C;
    out_bytes += 2.0 * jobs[i].L * jobs[i].Rp * jobs[i].Cp;
  }
  in_bytes = elems * sizeof(T);
  int64_t blocks1 = 0, blocks2 = 0;
  for (int i = 0; i < n; ++i) {
    const NormJob& j = jobs[i];
    const int flat = (j.sC == 1 && j.sR == j.C) ? 1 : 0;
    const int64_t ce = ps::norm_chunk_elems(j.R * j.C);
    int chunks = norm_chunks(j.L, j.R, j.C, sms);
    if (flat) chunks = static_cast<int>((j.R * j.C + ce - 1) / ce);
    for (ps::NormBatch* b : {&b1, &b2}) {
      ps::NormBatchProblem& q = b->p[i];
      q.x = j.x;
      q.xh = static_cast<__half*>(j.xh);
      q.partial = j.partial;
      q.R = j.R;
      q.C = j.C;
      q.sL = j.sL;
      q.sR = j.sR;
      q.sC = j.sC;
      q.Rp = j.Rp;
      q.Cp = j.Cp;
      q.chunk_elems = ce;
      q.flat = flat;
      q.chunks = chunks;
    }
    b1.p[i].b0 = blocks1;
    b1.p[i].per = chunks;
    blocks1 += j.L * chunks;
    // About 4 blocks per SM over the whole launch, shared by element count.
    const int64_t per_mat = (j.Rp * j.Cp + ps::NORM_THREADS * 8 - 1) / (ps::NORM_THREADS * 8);
    const double share = static_cast<double>(j.L) * j.R * j.C / elems;
    int64_t gx = static_cast<int64_t>(std::ceil(4.0 * sms * share / j.L));
    if (gx > per_mat) gx = per_mat;
    if (gx < 1) gx = 1;
    b2.p[i].b0 = blocks2;
    b2.p[i].per = gx;
    blocks2 += j.L * gx;
  }
  if (blocks1 > INT32_MAX || blocks2 > INT32_MAX)
    return fail(PS_ERR_INVALID, "ps_circuit: normalisation grid too large");
  {
    LaunchScope scope(kProfNormalize, s, 2.0 * elems, in_bytes);
    ps::ps_norm_partial_batched_kernel<T>
        <<<static_cast<unsigned>(blocks1), ps::NORM_THREADS, 0, s>>>(b1);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "normalize launch (batched pass 1)");
  }
  LaunchScope scope(kProfNormalize, s, elems, in_bytes + out_bytes);
  ps::ps_scale_cast_batched_kernel<T><<<static_cast<unsigned>(blocks2), ps::NORM_THREADS, 0, s>>>(b2);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PS_OK : cuda_fail(e, "normalize launch (batched pass 2)");
}

// The normalisations of a grouped circuit: jobs of one input type are batched
// NORM_BATCH_MAX at a time; a type with a single job takes normalize_impl.
int normalize_jobs(const std::vector<NormJob>& jobs, float eps, int sms, cudaStream_t s) {
  if (!(eps > 0.f)) return fail(PS_ERR_INVALID, "ps_normalize: eps must be positive");
  for (const NormJob& j : jobs)
    if (elem_bytes(j.x_dtype) == 0) return fail(PS_ERR_INVALID, "ps_normalize: bad dtype");
  DeviceState* st = nullptr;
  int rc0 = device_state(&st);
  if (rc0) return rc0;
  for (int dt : {PS_F16, PS_BF16, PS_F32, PS_F64}) {
    int grid = 0;
    switch (dt) {
      case PS_F16: grid = norm_fused_grid<__half>(st, dt); break;
      case PS_BF16: grid = norm_fused_grid<__nv_bfloat16>(st, dt); break;
      case PS_F32: grid = norm_fused_grid<float>(st, dt); break;
      default: grid = norm_fused_grid<double>(st, dt); break;
    }
    std::vector<NormJob> same, fused;
    for (const NormJob& j : jobs) {
      if (j.x_dtype != dt) continue;
      if (norm_fused_ok(j, grid, elem_bytes(dt)))
        fused.push_back(j);
      else
        same.push_back(j);
    }
    for (size_t i0 = 0; i0 < fused.size(); i0 += ps::NORM_BATCH_MAX) {
      const int n = static_cast<int>(std::min<size_t>(fused.size() - i0, ps::NORM_BATCH_MAX));
      const NormJob* b = fused.data() + i0;
      int rc;
      switch (dt) {
        case PS_F16: rc = launch_normalize_fused<__half>(b, n, eps, st, grid, s); break;
        case PS_BF16: rc = launch_normalize_fused<__nv_bfloat16>(b, n, eps, st, grid, s); break;
        case PS_F32: rc = launch_normalize_fused<float>(b, n, eps, st, grid, s); break;
        default: rc = launch_normalize_fused<double>(b, n, eps, st, grid, s); break;
      }
      if (rc) return rc;
    }
    for (size_t i0 = 0; i0 < same.size(); i0 += ps::NORM_BATCH_MAX) {
      const int n = static_cast<int>(std::min<size_t>(same.size() - i0, ps::NORM_BATCH_MAX));
      const NormJob* b = same.data() + i0;
      int rc;
      if (n == 1) {
        rc = normalize_impl(b->x, b->x_dtype, b->L, b->R, b->C, b->sL, b->sR, b->sC, eps, b->xh,
                            b->Rp, b->Cp, b->partial, normalize_ws_bytes(b->L, b->R, b->C, sms), s);
      } else {
        switch (dt) {
          case PS_F16: rc = launch_normalize_batch<__half>(b, n, eps, sms, s); break;
          case PS_BF16: rc = launch_normalize_batch<__nv_bfloat16>(b, n, eps, sms, s); break;
          case PS_F32: rc = launch_normalize_batch<float>(b, n, eps, sms, s); break;
          default: rc = launch_normalize_batch<double>(b, n, eps, sms, s); break;
        }
      }
      if (rc) return rc;
    }
  }
  return PS_OK;
}

template <typename T>
int launch_copy_out(const void* xh, int64_t Rp, int64_t Cp, int64_t R, int64_t C, int64_t L,
                    void* y, int sms, cudaStream_t s) {
  int64_t blocks = (L * R * C + ps::NORM_THREADS - 1) / ps::NORM_THREADS;
  if (blocks > 8LL * sms) blocks = 8LL * sms;
  if (blocks < 1) blocks = 1;
  LaunchScope scope(kProfOther, s, 0.0, static_cast<double>(L) * R * C * (2.0 + sizeof(T)));
  ps::ps_copy_out_kernel<T><<<static_cast<unsigned>(blocks), ps::NORM_THREADS, 0, s>>>(
      static_cast<const __half*>(xh), Rp, Cp, R, C, L, static_cast<T*>(y));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PS_OK : cuda_fail(e, "copy-out launch");
}

int copy_out(const void* xh, int64_t Rp, int64_t Cp, int64_t R, int64_t C, int64_t L, void* y,
             int y_dtype, int sms, cudaStream_t s) {
  switch (y_dtype) {
    case PS_F16:
      return launch_copy_out<__half>(xh, Rp, Cp, R, C, L, y, sms, s);
    case PS_BF16:
      return launch_copy_out<__nv_bfloat16>(xh, Rp, Cp, R, C, L, y, sms, s);
    case PS_F32:
      return launch_copy_out<float>(xh, Rp, Cp, R, C, L, y, sms, s);
    default:
      return launch_copy_out<double>(xh, Rp, Cp, R, C, L, y, sms, s);
  }
}

// ------------------------------------------------------------------ circuit
struct CircuitLayout {
  int64_t Rp, Cp, n, m;
  bool tall;
  int64_t xh_bytes, buf_bytes, norm_bytes, total;
};

CircuitLayout circuit_layout(int64_t L, int64_t rows, int64_t cols, int buffers, int sms) {
  CircuitLayout c;
  c.Rp = round_up(rows, 8);
  c.Cp = round_up(cols, 8);
  c.tall = rows > cols;
  c.n = c.tall ? c.Cp : c.Rp;
  c.m = c.tall ? c.Rp : c.Cp;
  c.xh_bytes = round_up(L * c.Rp * c.Cp * 2, 256);
  c.buf_bytes = round_up(L * c.n * c.n * 2, 256);
  c.norm_bytes = normalize_ws_bytes(L, rows, cols, sms);
  c.total = 2 * c.xh_bytes + buffers * c.buf_bytes + c.norm_bytes;
  return c;
}

int validate_table(int n_outer, const float* residuals, const int32_t* n_steps,
                   const ps_step* steps, int buffers) {
  if (n_outer <= 0 || !residuals || !n_steps || !steps || buffers < 1)
    return fail(PS_ERR_INVALID, "ps_circuit: empty circuit");
  int off = 0;
  for (int t = 0; t < n_outer; ++t) {
    if (n_steps[t] <= 0 || !std::isfinite(residuals[t]))
      return fail(PS_ERR_INVALID,
                  "ps_circuit: each outer iteration needs a finite residual and at least one "
                  "inner iteration");
    unsigned initialized = 1u;  // B[0] holds the Gram matrix
    for (int s = 0; s < n_steps[t]; ++s) {
      const ps_step& p = steps[off + s];
      if (p.dst < 0 || p.src < 0 || p.add < 0 || p.dst >= buffers || p.src >= buffers ||
          p.add >= buffers || p.dst >= 32 || p.dst == p.src || !(initialized >> p.src & 1u) ||
          !(initialized >> p.add & 1u) || !std::isfinite(p.alpha) || !std::isfinite(p.beta) ||
          !std::isfinite(p.diag))
        return fail(PS_ERR_INVALID, "ps_circuit: invalid inner iteration %d of outer %d", s, t);
      initialized |= 1u << p.dst;
    }
    off += n_steps[t];
  }
  return PS_OK;
}

// Workspace layout of a grouped circuit: per problem two FP16 copies of X
// (padded to multiples of 8), the square buffers of all problems that share
// the same n stacked so one launch serves them all, and per-problem scratch
// for the normalisation partial sums.
struct GroupedPlan {
  struct Prob {
    CircuitLayout lay;
    int group;
    int64_t goff;          // first matrix of this problem inside its n-group
    int64_t xh_off[2];
    int64_t norm_off;
    int64_t cnt_off;  // L counters of the fused normalisation
  };
  struct NGroup {
    int64_t n, Ltot, buf_off, buf_bytes;
    int64_t ctr_off;  // per-matrix completion counters of chain launches
  };
  std::vector<Prob> probs;
  std::vector<NGroup> groups;
  int64_t ctr_off = 0, ctr_bytes = 0;  // all groups' counters, one contiguous range
  int64_t circ_off = 0;                 // whole-circuit kernel counters (inside that range)
  int64_t total = 0;
};

int make_grouped_plan(const ps_problem* probs, int n_probs, int buffers, int sms,
                      GroupedPlan* plan) {
  if (!probs || n_probs <= 0 || n_probs > 4096)
    return fail(PS_ERR_INVALID, "ps_circuit: bad problem list");
  if (buffers < 1 || buffers > 32) return fail(PS_ERR_INVALID, "ps_circuit: bad buffer count");
  plan->probs.resize(n_probs);
  int64_t off = 0;
  for (int i = 0; i < n_probs; ++i) {
    const ps_problem& q = probs[i];
    if (!dims_ok(q.L, q.rows, q.cols)) return fail(PS_ERR_INVALID, "ps_circuit: bad sizes (problem %d)", i);
    GroupedPlan::Prob& p = plan->probs[i];
    p.lay = circuit_layout(q.L, q.rows, q.cols, buffers, sms);
    int g = -1;
    for (size_t k = 0; k < plan->groups.size(); ++k)
      if (plan->groups[k].n == p.lay.n) g = static_cast<int>(k);
    if (g < 0) {
      plan->groups.push_back({p.lay.n, 0, 0, 0, 0});
      g = static_cast<int>(plan->groups.size()) - 1;
    }
    p.group = g;
    p.goff = plan->groups[g].Ltot;
    plan->groups[g].Ltot += q.L;
    p.xh_off[0] = off;
    p.xh_off[1] = off + p.lay.xh_bytes;
    off += 2 * p.lay.xh_bytes;
  }
  for (GroupedPlan::NGroup& g : plan->groups) {
    g.buf_bytes = round_up(g.Ltot * g.n * g.n * 2, 256);
    g.buf_off = off;
    off += buffers * g.buf_bytes;
  }
  for (GroupedPlan::Prob& p : plan->probs) {
    p.norm_off = off;
    off += p.lay.norm_bytes;
  }
  plan->ctr_off = off;
  for (GroupedPlan::NGroup& g : plan->groups) {
    g.ctr_off = off;
    off += round_up(g.Ltot * static_cast<int64_t>(sizeof(unsigned)), 256);
  }
  for (int i = 0; i < n_probs; ++i) {
    plan->probs[i].cnt_off = off;
    off += round_up(probs[i].L * static_cast<int64_t>(sizeof(unsigned)), 256);
  }
  int64_t ltot = 0;
  for (int i = 0; i < n_probs; ++i) ltot += probs[i].L;
  plan->circ_off = off;  // whole-circuit kernel: one counter per matrix of every problem
  off += round_up(ltot * static_cast<int64_t>(sizeof(unsigned)), 256);
  plan->ctr_bytes = off - plan->ctr_off;
  plan->total = off;
  return PS_OK;
}

// ------------------------------------------------------------------ whole circuit
// Whether a grouped circuit runs as one ps_circuit_pair_kernel launch: the
// CTA-pair path for every problem and the kernel's table limits.
bool use_circuit_kernel(const GroupedPlan& plan, int n_probs, int n_outer, const int32_t* n_steps,
                        int buffers) {
  if (!g_circuit_mode || n_probs > ps::circ::MAXP || buffers > ps::circ::MAXB) return false;
  int stages = 0, steps = 0;
  for (int t = 0; t < n_outer; ++t) {
    stages += n_steps[t] + 2;
    steps += n_steps[t];
  }
  if (stages > ps::circ::MAX_STAGES || steps > ps::circ::MAX_STEPS) return false;
  for (const GroupedPlan::Prob& p : plan.probs)
    if (!use_pair(true, p.lay.n) || !use_pair(false, p.lay.n)) return false;
  // the item table indexes matrices with 16 bits
  for (const GroupedPlan::NGroup& g : plan.groups)
    if (g.Ltot > 65535) return false;
  return true;
}

// Where a whole-circuit launch also stores its final results (other GPUs'
// copies of the buffer holding every y, at peer_bases[k] for the buffer at
// local_base here) and how its matrices are ordered: phase_ends[i * n_phases +
// k] is the number of problem i's matrices in phases 0..k; the tiles of a
// phase are scheduled before those of the next, so its results are final
// (and pushed) while later phases compute. No push and one phase: nullptr.
struct CircuitPush {
  const uint8_t* local_base = nullptr;
  const void* const* peer_bases = nullptr;
  int n_peers = 0;
  int n_phases = 1;
  const int32_t* phase_ends = nullptr;
  unsigned* sig = nullptr;  // phase flags, counters and exit count (see CircuitParams)
};

// All stages of a grouped circuit in one launch (ps_circuit.cuh). `cur0` is
// the Xh buffer holding the normalised inputs; the final applies store into
// y (direct problems) or Xh[1 - final cur] (the caller copies those out).
int circuit_kernel_run(const GroupedPlan& plan, const ps_problem* probs, const ps_update* updates,
                       int n_probs, int n_outer, const float* residuals, const int32_t* n_steps,
                       const ps_step* steps, int buffers, uint8_t* ws, const std::vector<bool>& direct,
                       cudaStream_t stream, const CircuitPush* push = nullptr) {
  using ps::circ::CircuitParams;
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  auto kern = ps::circ::ps_circuit_pair_kernel;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(ps::pair::NUM_THREADS);
  cfg.dynamicSmemBytes = ps::pair::SMEM_TOTAL;
  cfg.stream = stream;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  if (!st->circ_ready) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         ps::pair::SMEM_TOTAL);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(circuit smem)");
    cfg.gridDim = dim3(2 * (st->sms / 2));
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters(circuit)");
    if (clusters < 1) return fail(PS_ERR_UNSUPPORTED, "no co-resident CTA pair fits on the device");
    st->circ_clusters = clusters;
    st->circ_ready = true;
  }
  static thread_local CircuitParams P;
  std::memset(&P, 0, sizeof(P));
  // stage table
  int ns = 0, off = 0, nsym = 0, napp = 0;
  for (int t = 0; t < n_outer; ++t) {
    auto add_stage = [&](int kind, int step) {
      P.st_kind[ns] = static_cast<unsigned char>(kind);
      P.st_t[ns] = static_cast<unsigned char>(t);
      P.st_step[ns] = static_cast<unsigned char>(step);
      P.st_nsym[ns] = static_cast<unsigned char>(nsym);
      P.st_napp[ns] = static_cast<unsigned char>(napp);
      ++ns;
      if (kind == ps::circ::kApply)
        ++napp;
      else
        ++nsym;
    };
    add_stage(ps::circ::kGram, 0);
    for (int k = 0; k < n_steps[t]; ++k) add_stage(ps::circ::kSquare, off + k);
    add_stage(ps::circ::kApply, off + n_steps[t] - 1);
    P.residual[t] = residuals[t];
    off += n_steps[t];
  }
  for (int i = 0; i < off; ++i)
    P.steps[i] = {steps[i].dst, steps[i].src, steps[i].add, steps[i].alpha, steps[i].beta,
                  steps[i].diag};
  P.n_outer = n_outer;
  P.n_stages = ns;
  P.nprob = n_probs;
  int pairs = st->circ_clusters;
  if (g_max_ctas > 1 && pairs > g_max_ctas / 2) pairs = g_max_ctas / 2;
  // per problem: maps, shapes, tiles, chunking
  std::vector<int64_t> total_per_mat(n_probs);
  int64_t g0 = 0;
  for (int i = 0; i < n_probs; ++i) {
    const GroupedPlan::Prob& p = plan.probs[i];
    const GroupedPlan::NGroup& g = plan.groups[p.group];
    const ps_problem& q = probs[i];
    ps::circ::CProblem& c = P.prob[i];
    const int64_t Rp = p.lay.Rp, Cp = p.lay.Cp, n = p.lay.n, L = q.L;
    int ck = 0, ck2 = 0;
    for (int x = 0; x < 2; ++x) {
      uint8_t* xh = ws + p.xh_off[x];
      if ((rc = map_pair_operand(&c.xk[x], xh, false, Cp, Rp, L, Cp, Rp * Cp, &ck))) return rc;
      if ((rc = map_pair_operand(&c.xm[x], xh, true, Cp, Rp, L, Cp, Rp * Cp, &ck2))) return rc;
      if ((rc = map_out(&c.xo[x], xh, PS_F16, Cp, Rp, L, Cp, Rp * Cp))) return rc;
      c.xh[x] = reinterpret_cast<const __half*>(xh);
    }
    if (ck != ck2) return fail(PS_ERR_INVALID, "internal: X maps disagree on the chunked layout");
    c.ck_x = ck;
    for (int k = 0; k < buffers; ++k) {
      uint8_t* bp = ws + g.buf_off + k * g.buf_bytes + p.goff * n * n * 2;
      if ((rc = map_pair_operand(&c.bk[k], bp, false, n, n, L, n, n * n, &ck))) return rc;
      if ((rc = map_pair_operand(&c.bm[k], bp, true, n, n, L, n, n * n, &ck2))) return rc;
      if ((rc = map_out(&c.bo[k], bp, PS_F16, n, n, L, n, n * n))) return rc;
      c.buf[k] = reinterpret_cast<const __half*>(bp);
    }
    if (ck != ck2) return fail(PS_ERR_INVALID, "internal: buffer maps disagree on the chunked layout");
    c.ck_b = ck;
    const bool upd = updates && updates[i].p;
    c.direct = direct[i] ? 1 : 0;
    c.y_out = q.y_dtype == PS_F32 ? ps::kOutF32 : q.y_dtype == PS_BF16 ? ps::kOutBF16 : ps::kOutF16;
    if (direct[i] && !upd) {
      if ((rc = map_out(&c.yo, q.y, q.y_dtype, q.cols, q.rows, L, q.cols, q.rows * q.cols))) return rc;
      c.y = static_cast<unsigned char*>(q.y);
    }
    if (upd) {
      c.upd = 1;
      c.p_dtype = updates[i].p_dtype == PS_F32 ? ps::kOutF32
                  : updates[i].p_dtype == PS_BF16 ? ps::kOutBF16 : ps::kOutF16;
      c.P = updates[i].p;
      c.decay = updates[i].decay;
      c.upd_alpha = updates[i].alpha;
    }
    c.L = static_cast<int>(L);
    c.Rp = static_cast<int>(Rp);
    c.Cp = static_cast<int>(Cp);
    c.n = static_cast<int>(n);
    c.m = static_cast<int>(p.lay.m);
    c.tall = p.lay.tall ? 1 : 0;
    c.Tsym = pair_sym_tiles(n);
    const int64_t M = p.lay.tall ? p.lay.m : n, N = p.lay.tall ? n : p.lay.m;
    c.tiles_m2 = static_cast<int>((M + 255) / 256);
    c.tiles_n = static_cast<int>((N + 255) / 256);
    c.g0 = static_cast<int>(g0);
    g0 += L;
    total_per_mat[i] = static_cast<int64_t>(nsym) * c.Tsym + static_cast<int64_t>(napp) * c.tiles_m2 * c.tiles_n;
  }
  // Chunks: a round (every stage of one chunk per problem, skewed) should hold
  // about two waves of pair tiles, so a tile's inputs were scheduled a round
  // earlier; grown uniformly until the item table fits.
  // Phases (push): matrices [begin(i, k), end(i, k)) of problem i in phase k.
  const int n_phases = push ? push->n_phases : 1;
  auto phase_begin = [&](int i, int k) -> int64_t {
    return k == 0 ? 0 : static_cast<int64_t>(push->phase_ends[i * n_phases + k - 1]);
  };
  auto phase_end = [&](int i, int k) -> int64_t {
    return n_phases == 1 ? probs[i].L : static_cast<int64_t>(push->phase_ends[i * n_phases + k]);
  };
  std::vector<int64_t> C(n_probs);
  for (int i = 0; i < n_probs; ++i) {
    C[i] = (2LL * pairs + total_per_mat[i] - 1) / total_per_mat[i];
    if (C[i] < 1) C[i] = 1;
    if (C[i] > probs[i].L) C[i] = probs[i].L;
  }
  auto chunks_of = [&](int i, int k) { return (phase_end(i, k) - phase_begin(i, k) + C[i] - 1) / C[i]; };
  auto count_items = [&]() {
    int64_t items = 0;
    for (int k = 0; k < n_phases; ++k)
      for (int i = 0; i < n_probs; ++i) items += ns * chunks_of(i, k);
    return items;
  };
  while (count_items() > ps::circ::MAX_ITEMS) {
    bool grew = false;
    for (int i = 0; i < n_probs; ++i)
      if (C[i] < probs[i].L) {
        C[i] = std::min<int64_t>(probs[i].L, C[i] * 2);
        grew = true;
      }
    if (!grew) return fail(PS_ERR_UNSUPPORTED, "circuit kernel: item table too large");
  }
  for (int i = 0; i < n_probs; ++i) P.prob[i].chunk = static_cast<int>(C[i]);
  int items = 0;
  int64_t tiles = 0;
  for (int k = 0; k < n_phases; ++k) {
    int64_t max_nch = 0;
    for (int i = 0; i < n_probs; ++i) max_nch = std::max<int64_t>(max_nch, chunks_of(i, k));
    for (int64_t round = 0; round < max_nch + ns - 1; ++round)
      for (int i = 0; i < n_probs; ++i) {
        const int64_t nch = chunks_of(i, k), b0 = phase_begin(i, k), b1 = phase_end(i, k);
        for (int sg = 0; sg < ns; ++sg) {
          const int64_t c = round - sg;
          if (c < 0 || c >= nch) continue;
          const int64_t first = b0 + c * C[i];
          P.item_start[items] = static_cast<int>(tiles);
          P.item_stage[items] = static_cast<unsigned char>(sg);
          P.item_prob[items] = static_cast<unsigned char>(i);
          P.item_first[items] = static_cast<unsigned short>(first);
          P.item_phase[items] = static_cast<unsigned char>(k);
          ++items;
          const int64_t size = std::min<int64_t>(C[i], b1 - first);
          const int per = P.st_kind[sg] == ps::circ::kApply ? P.prob[i].tiles_m2 * P.prob[i].tiles_n
                                                            : P.prob[i].Tsym;
          tiles += size * per;
          if (sg == ns - 1)
            P.sig_target[k] += static_cast<unsigned>(size * per * ps::circ::SIGNALS_PER_TILE);
        }
      }
  }
  if (push && push->sig) {
    P.sig = push->sig;
    P.n_sig = n_phases;
  }
  if (push) {
    P.n_peers = push->n_peers;
    for (int k = 0; k < push->n_peers; ++k)
      P.peer_delta[k] = static_cast<long long>(reinterpret_cast<uintptr_t>(push->peer_bases[k]) -
                                               reinterpret_cast<uintptr_t>(push->local_base));
  }
  if (tiles > INT32_MAX) return fail(PS_ERR_UNSUPPORTED, "circuit kernel: too many tiles");
  P.item_start[items] = static_cast<int>(tiles);
  P.n_items = items;
  P.total_tiles = static_cast<int>(tiles);
  P.done = reinterpret_cast<unsigned*>(ws + plan.circ_off);
  P.status = st->status;
  P.wait_limit = g_wait_limit;
  if (pairs > P.total_tiles) pairs = P.total_tiles;
  cfg.gridDim = dim3(2 * pairs);
  double flops = 0.0;
  for (int i = 0; i < n_probs; ++i) {
    const double n = static_cast<double>(plan.probs[i].lay.n), m = static_cast<double>(plan.probs[i].lay.m);
    flops += probs[i].L * (n_outer * 3.0 * n * n * m + off * n * n * n);
  }
  LaunchScope scope(kProfCircuit, stream, flops, 0.0);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, P);
  if (e != cudaSuccess) return cuda_fail(e, "circuit kernel launch");
  return PS_OK;
}

template <typename T, typename TO>
int launch_muon_direction(const void* const* grads, void* const* moms, int count, int64_t E,
                          float mu, int nesterov, void* out, int sms, cudaStream_t s) {
  for (int i0 = 0; i0 < count; i0 += ps::MUON_MAX_PARAMS) {
    const int n = count - i0 < ps::MUON_MAX_PARAMS ? count - i0 : ps::MUON_MAX_PARAMS;
    ps::MuonDirectionArgs a;
    std::memset(&a, 0, sizeof(a));
    for (int i = 0; i < n; ++i) {
      a.grad[i] = grads[i0 + i];
      a.mom[i] = moms[i0 + i];
    }
    a.E = E;
    a.mu = mu;
    a.nesterov = nesterov;
    TO* o = static_cast<TO*>(out) + static_cast<int64_t>(i0) * E;
    bool vec = E % 8 == 0 && aligned16(o);
    for (int i = 0; i < n && vec; ++i) vec = aligned16(a.grad[i]) && aligned16(a.mom[i]);
    int64_t gx = (E + ps::NORM_THREADS * (vec ? 8 : 4) - 1) / (ps::NORM_THREADS * (vec ? 8 : 4));
    const int64_t cap = (8LL * sms + n - 1) / n;
    if (gx > cap) gx = cap;
    if (gx < 1) gx = 1;
    LaunchScope scope(kProfOther, s, 3.0 * n * E, static_cast<double>(n) * E * (3.0 * sizeof(T) + sizeof(TO)));
    const dim3 grid(static_cast<unsigned>(gx), n);
    if (vec)
      ps::ps_muon_direction_kernel<T, TO, 8><<<grid, ps::NORM_THREADS, 0, s>>>(a, o);
    else
      ps::ps_muon_direction_kernel<T, TO, 1><<<grid, ps::NORM_THREADS, 0, s>>>(a, o);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "muon direction launch");
  }
  return PS_OK;
}

template <typename T>
int muon_direction_out(int out_dtype, const void* const* grads, void* const* moms, int count, int64_t E,
                       float mu, int nesterov, void* out, int sms, cudaStream_t s) {
  switch (out_dtype) {
    case PS_F16:
      return launch_muon_direction<T, __half>(grads, moms, count, E, mu, nesterov, out, sms, s);
    case PS_BF16:
      return launch_muon_direction<T, __nv_bfloat16>(grads, moms, count, E, mu, nesterov, out, sms, s);
    default:
      return launch_muon_direction<T, float>(grads, moms, count, E, mu, nesterov, out, sms, s);
  }
}
template <typename T, typename TU>
int launch_muon_update(void* const* params, int count, int64_t E, float decay, float alpha,
                       const void* upd, int sms, cudaStream_t s) {
  for (int i0 = 0; i0 < count; i0 += ps::MUON_MAX_PARAMS) {
    const int n = count - i0 < ps::MUON_MAX_PARAMS ? count - i0 : ps::MUON_MAX_PARAMS;
    ps::MuonUpdateArgs a;
    std::memset(&a, 0, sizeof(a));
    for (int i = 0; i < n; ++i) a.param[i] = params[i0 + i];
    a.E = E;
    a.decay = decay;
    a.alpha = alpha;
    const TU* u = static_cast<const TU*>(upd) + static_cast<int64_t>(i0) * E;
    bool vec = E % 8 == 0 && aligned16(u);
    for (int i = 0; i < n && vec; ++i) vec = aligned16(a.param[i]);
    int64_t gx = (E + ps::NORM_THREADS * (vec ? 8 : 4) - 1) / (ps::NORM_THREADS * (vec ? 8 : 4));
    const int64_t cap = (8LL * sms + n - 1) / n;
    if (gx > cap) gx = cap;
    if (gx < 1) gx = 1;
    LaunchScope scope(kProfOther, s, 3.0 * n * E, static_cast<double>(n) * E * (2.0 * sizeof(T) + sizeof(TU)));
    const dim3 grid(static_cast<unsigned>(gx), n);
    if (vec)
      ps::ps_muon_update_kernel<T, TU, 8><<<grid, ps::NORM_THREADS, 0, s>>>(a, u);
    else
      ps::ps_muon_update_kernel<T, TU, 1><<<grid, ps::NORM_THREADS, 0, s>>>(a, u);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "muon update launch");
  }
  return PS_OK;
}

template <typename T>
int muon_update_in(int upd_dtype, void* const* params, int count, int64_t E, float decay, float alpha,
                   const void* upd, int sms, cudaStream_t s) {
  switch (upd_dtype) {
    case PS_F16:
      return launch_muon_update<T, __half>(params, count, E, decay, alpha, upd, sms, s);
    case PS_BF16:
      return launch_muon_update<T, __nv_bfloat16>(params, count, E, decay, alpha, upd, sms, s);
    default:
      return launch_muon_update<T, float>(params, count, E, decay, alpha, upd, sms, s);
  }
}

// NaN / infinity counts and max |x| per matrix, matrices of E contiguous
// elements; outputs zeroed here, on the stream, before the kernel.
template <typename T>
int launch_update_stats(const void* x, int64_t L, int64_t E, int64_t* nan_count, int64_t* inf_count,
                        float* max_abs, int sms, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(nan_count, 0, L * sizeof(int64_t), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(inf_count, 0, L * sizeof(int64_t), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(max_abs, 0, L * sizeof(float), s);
  if (e != cudaSuccess) return cuda_fail(e, "update stats memset");
  const int64_t per_mat = (E + ps::NORM_THREADS * 8 - 1) / (ps::NORM_THREADS * 8);
  for (int64_t l0 = 0; l0 < L; l0 += kMaxGridY) {  // matrices run along grid y
    const int64_t n = L - l0 < kMaxGridY ? L - l0 : kMaxGridY;
    int64_t gx = (4LL * sms + n - 1) / n;
    if (gx > per_mat) gx = per_mat;
    if (gx < 1) gx = 1;
    LaunchScope scope(kProfOther, s, 0.0, static_cast<double>(n) * E * sizeof(T));
    ps::ps_update_stats_kernel<T><<<dim3(static_cast<unsigned>(gx), static_cast<unsigned>(n)),
                                    ps::NORM_THREADS, 0, s>>>(
        static_cast<const T*>(x) + l0 * E, E,
        reinterpret_cast<unsigned long long*>(nan_count + l0),
        reinterpret_cast<unsigned long long*>(inf_count + l0),
        reinterpret_cast<unsigned int*>(max_abs + l0));
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "update stats launch");
  }
  return PS_OK;
}

}  // namespace

// ====================================================================== C ABI
extern "C" {

int ps_version(void) { return kVersion; }

const char* ps_last_error(void) { return g_last_error.c_str(); }

int ps_get_status(int* status, int clear) {
  if (!status) return fail(PS_ERR_INVALID, "ps_get_status: null pointer");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  cudaError_t e = cudaMemcpy(status, st->status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read status");
  if (clear) {
    e = cudaMemset(st->status, 0, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "clear status");
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "clear status");
  }
  return PS_OK;
}

long long ps_launch_count(void) { return g_launches.load(); }

int ps_profile_enable(int enable) {
  std::lock_guard<std::mutex> lock(g_prof_mu);
  if (enable) {
    for (ProfRecord& r : g_prof) {
      g_event_pool.push_back(r.start);
      g_event_pool.push_back(r.stop);
    }
    g_prof.clear();
  }
  g_prof_on = enable != 0;
  return PS_OK;
}

int ps_profile_read(int kind, double* total_ms, int64_t* launches, double* flops, double* bytes) {
  if (kind < 0 || kind >= kNumProfKinds || !total_ms || !launches || !flops || !bytes)
    return fail(PS_ERR_INVALID, "ps_profile_read: bad arguments");
  std::lock_guard<std::mutex> lock(g_prof_mu);
  double ms = 0.0, f = 0.0, b = 0.0;
  int64_t n = 0;
  for (const ProfRecord& r : g_prof) {
    if (r.kind != kind) continue;
    cudaError_t e = cudaEventSynchronize(r.stop);
    if (e != cudaSuccess) return cuda_fail(e, "ps_profile_read");
    float t = 0.f;
    e = cudaEventElapsedTime(&t, r.start, r.stop);
    if (e != cudaSuccess) return cuda_fail(e, "ps_profile_read");
    ms += t;
    f += r.flops;
    b += r.bytes;
    ++n;
  }
  *total_ms = ms;
  *launches = n;
  *flops = f;
  *bytes = b;
  return PS_OK;
}

int ps_set_max_ctas(int max_ctas) {
  if (max_ctas < 0) return fail(PS_ERR_INVALID, "ps_set_max_ctas: negative limit");
  const int previous = g_max_ctas;
  g_max_ctas = max_ctas;
  return previous;
}

int ps_set_cta_pairs(int mode) {
  if (mode < 0 || mode > 2) return fail(PS_ERR_INVALID, "ps_set_cta_pairs: mode must be 0, 1 or 2");
  const int previous = g_pair_mode;
  g_pair_mode = mode;
  return previous;
}

int ps_set_fused_normalize(int mode) {
  if (mode < 0 || mode > 1)
    return fail(PS_ERR_INVALID, "ps_set_fused_normalize: mode must be 0 or 1");
  const int previous = g_norm_fused;
  g_norm_fused = mode;
  return previous;
}

int ps_set_circuit_kernel(int mode) {
  if (mode < 0 || mode > 1) return fail(PS_ERR_INVALID, "ps_set_circuit_kernel: mode must be 0 or 1");
  const int previous = g_circuit_mode;
  g_circuit_mode = mode;
  return previous;
}

int ps_set_chain(int mode) {
  if (mode < 0 || mode > 1) return fail(PS_ERR_INVALID, "ps_set_chain: mode must be 0 or 1");
  const int previous = g_chain_mode;
  g_chain_mode = mode;
  return previous;
}

int ps_set_wait_limit(long long cycles) {
  if (cycles <= 0) return fail(PS_ERR_INVALID, "ps_set_wait_limit: cycles must be positive");
  g_wait_limit = cycles;
  return PS_OK;
}

int ps_selftest_wait(long long limit_cycles, void* stream) {
  if (limit_cycles <= 0) return fail(PS_ERR_INVALID, "ps_selftest_wait: limit must be positive");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  ps::ps_selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(st->status,
                                                                               limit_cycles);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PS_OK : cuda_fail(e, "selftest launch");
}

int ps_selftest_chain_wait(void* workspace, int64_t workspace_bytes, long long limit_cycles,
                           void* stream) {
  if (!workspace || !aligned16(workspace))
    return fail(PS_ERR_INVALID, "ps_selftest_chain_wait: null or misaligned workspace");
  if (workspace_bytes < PS_SELFTEST_CHAIN_WORKSPACE_BYTES)
    return fail(PS_ERR_WORKSPACE, "ps_selftest_chain_wait: workspace too small");
  if (limit_cycles <= 0 || limit_cycles > g_wait_limit / 4)
    return fail(PS_ERR_INVALID, "ps_selftest_chain_wait: limit must be positive and at most a "
                                "quarter of the wait limit");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Two 256 x 256 matrices, two buffers, two inner iterations; the counters
  // start far below what step 1 waits for, so every step-1 tile's wait runs
  // out (after limit_cycles, before any mbarrier wait could).
  const int64_t n = 256, L = 2, buf_bytes = L * n * n * 2;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  cudaError_t e = cudaMemsetAsync(ws, 0, 2 * buf_bytes + 256, s);
  if (e != cudaSuccess) return cuda_fail(e, "ps_selftest_chain_wait memset");
  const ps_step steps[2] = {{1, 0, 0, 1.f, 0.f, 0.f}, {0, 1, 1, 1.f, 0.f, 0.f}};
  return chain_launch(ws, buf_bytes, 2, L, n, steps, 2,
                      reinterpret_cast<unsigned*>(ws + 2 * buf_bytes), 0x40000000u, s, limit_cycles);
}

int64_t ps_normalize_workspace_bytes(int64_t L, int64_t rows, int64_t cols) {
  DeviceState* st = nullptr;
  if (device_state(&st)) return -1;
  if (!dims_ok(L, rows, cols)) return -1;
  return normalize_ws_bytes(L, rows, cols, st->sms);
}

int ps_normalize(const void* x, int x_dtype, int64_t L, int64_t rows, int64_t cols, int64_t sL,
                 int64_t sR, int64_t sC, float eps, void* xh, int64_t rows_p, int64_t cols_p,
                 void* workspace, int64_t workspace_bytes, void* stream) {
  return normalize_impl(x, x_dtype, L, rows, cols, sL, sR, sC, eps, xh, rows_p, cols_p,
                        workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int ps_sumsq(const void* x, int x_dtype, int64_t L, int64_t rows, int64_t cols, int64_t sL,
             int64_t sR, int64_t sC, double* sums, void* workspace, int64_t workspace_bytes,
             void* stream) {
  if (!x || !sums || !workspace) return fail(PS_ERR_INVALID, "ps_sumsq: null pointer");
  if (!dims_ok(L, rows, cols)) return fail(PS_ERR_INVALID, "ps_sumsq: bad sizes");
  if (elem_bytes(x_dtype) == 0) return fail(PS_ERR_INVALID, "ps_sumsq: bad dtype");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  if (workspace_bytes < normalize_ws_bytes(L, rows, cols, st->sms))
    return fail(PS_ERR_WORKSPACE, "ps_sumsq: workspace too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  double* partial = static_cast<double*>(workspace);
  const int chunks = norm_chunks(L, rows, cols, st->sms);
  const int64_t ce = ps::norm_chunk_elems(rows * cols);
  int nch = 0;
  switch (x_dtype) {
    case PS_F16:
      rc = launch_norm_pass1<__half>(x, L, rows, cols, sL, sR, sC, partial, chunks, ce, &nch, s);
      break;
    case PS_BF16:
      rc = launch_norm_pass1<__nv_bfloat16>(x, L, rows, cols, sL, sR, sC, partial, chunks, ce, &nch, s);
      break;
    case PS_F32:
      rc = launch_norm_pass1<float>(x, L, rows, cols, sL, sR, sC, partial, chunks, ce, &nch, s);
      break;
    default:
      rc = launch_norm_pass1<double>(x, L, rows, cols, sL, sR, sC, partial, chunks, ce, &nch, s);
  }
  if (rc) return rc;
  const int64_t blocks = (L + 7) / 8;
  LaunchScope scope(kProfOther, s, 0.0, 8.0 * L * nch);
  ps::ps_sum_partials_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(partial, nch, L, sums);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? PS_OK : cuda_fail(e, "sum-of-squares launch");
}

int ps_scale_cast(const void* x, int x_dtype, int64_t L, int64_t rows, int64_t cols, int64_t sL,
                  int64_t sR, int64_t sC, const double* sums, float eps, void* xh, int64_t rows_p,
                  int64_t cols_p, void* stream) {
  if (!x || !xh) return fail(PS_ERR_INVALID, "ps_scale_cast: null pointer");
  if (!dims_ok(L, rows, cols) || rows_p < rows || cols_p < cols)
    return fail(PS_ERR_INVALID, "ps_scale_cast: bad sizes");
  if (elem_bytes(x_dtype) == 0) return fail(PS_ERR_INVALID, "ps_scale_cast: bad dtype");
  if (!std::isfinite(eps) || eps < 0.f)
    return fail(PS_ERR_INVALID, "ps_scale_cast: eps must be finite and non-negative");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (x_dtype) {
    case PS_F16:
      return launch_norm_pass2<__half>(x, L, rows, cols, sL, sR, sC, sums, 1, eps, xh, rows_p, cols_p,
                                       st->sms, s);
    case PS_BF16:
      return launch_norm_pass2<__nv_bfloat16>(x, L, rows, cols, sL, sR, sC, sums, 1, eps, xh, rows_p,
                                              cols_p, st->sms, s);
    case PS_F32:
      return launch_norm_pass2<float>(x, L, rows, cols, sL, sR, sC, sums, 1, eps, xh, rows_p, cols_p,
                                      st->sms, s);
    default:
      return launch_norm_pass2<double>(x, L, rows, cols, sL, sR, sC, sums, 1, eps, xh, rows_p, cols_p,
                                       st->sms, s);
  }
}

int ps_gram_f32(const void* x, float* out, int64_t L, int64_t rows, int64_t cols, int64_t x_ld,
                void* stream) {
  if (!x || !out) return fail(PS_ERR_INVALID, "ps_gram_f32: null pointer");
  if (!dims_ok(L, rows, cols) || x_ld < cols) return fail(PS_ERR_INVALID, "ps_gram_f32: bad sizes");
  if (x_ld % 8) return fail(PS_ERR_INVALID, "ps_gram_f32: x_ld must be a multiple of 8");
  if (!aligned16(x) || !aligned16(out))
    return fail(PS_ERR_INVALID, "ps_gram_f32: pointers must be 16-byte aligned");
  const bool tall = rows > cols;
  const int64_t n = tall ? cols : rows, K = tall ? rows : cols;
  if (n % 8) return fail(PS_ERR_INVALID, "ps_gram_f32: min(rows, cols) must be a multiple of 8");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap ta, tb, td;
  int rc;
  if ((rc = map_out(&td, out, PS_F32, n, n, L, n, n * n))) return rc;
  // The full n x n product on general tiles, FP32 out: no rounding, so the
  // sum of such partial Grams can be rounded once.
  ps::GemmArgs a = base_args(n, n, K, L);
  fill_gen_tiles(a, n, n, L);
  const double flops = 2.0 * L * n * n * K;
  const double bytes = static_cast<double>(L) * (2.0 * n * K + 4.0 * n * n);
  if (!tall) {
    if ((rc = map_kmajor(&ta, x, K, n, L, x_ld, rows * x_ld, ps::BM))) return rc;
    if ((rc = map_kmajor(&tb, x, K, n, L, x_ld, rows * x_ld, b_box_rows(false)))) return rc;
    return launch_gemm<false, false, false, ps::kOutF32>(9, ta, tb, td, a, s, kProfGram, flops, bytes,
                                                         false);
  }
  if ((rc = map_mnmajor(&ta, x, n, K, L, x_ld, rows * x_ld))) return rc;
  return launch_gemm<true, true, false, ps::kOutF32>(10, ta, ta, td, a, s, kProfGram, flops, bytes,
                                                     false);
}

int ps_muon_direction(const void* const* grads, void* const* moms, int count, int64_t elems,
                      int dtype, float mu, int nesterov, void* out, int out_dtype, void* stream) {
  if (!grads || !moms || !out) return fail(PS_ERR_INVALID, "ps_muon_direction: null pointer");
  if (count < 1 || elems < 1) return fail(PS_ERR_INVALID, "ps_muon_direction: empty bucket");
  for (int i = 0; i < count; ++i)
    if (!grads[i] || !moms[i]) return fail(PS_ERR_INVALID, "ps_muon_direction: null matrix %d", i);
  if (dtype != PS_F32 && dtype != PS_BF16 && dtype != PS_F16)
    return fail(PS_ERR_INVALID, "ps_muon_direction: parameters must be FP32, BF16 or FP16");
  if (out_dtype != PS_F32 && out_dtype != PS_BF16 && out_dtype != PS_F16)
    return fail(PS_ERR_INVALID, "ps_muon_direction: the output must be FP32, BF16 or FP16");
  if (!std::isfinite(mu)) return fail(PS_ERR_INVALID, "ps_muon_direction: momentum must be finite");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PS_F32:
      return muon_direction_out<float>(out_dtype, grads, moms, count, elems, mu, nesterov, out, st->sms, s);
    case PS_BF16:
      return muon_direction_out<__nv_bfloat16>(out_dtype, grads, moms, count, elems, mu, nesterov, out,
                                               st->sms, s);
    default:
      return muon_direction_out<__half>(out_dtype, grads, moms, count, elems, mu, nesterov, out, st->sms, s);
  }
}

int ps_muon_update(void* const* params, int count, int64_t elems, int dtype, const void* updates,
                   int upd_dtype, float decay, float alpha, void* stream) {
  if (!params || !updates) return fail(PS_ERR_INVALID, "ps_muon_update: null pointer");
  if (count < 1 || elems < 1) return fail(PS_ERR_INVALID, "ps_muon_update: empty bucket");
  for (int i = 0; i < count; ++i)
    if (!params[i]) return fail(PS_ERR_INVALID, "ps_muon_update: null matrix %d", i);
  if (dtype != PS_F32 && dtype != PS_BF16 && dtype != PS_F16)
    return fail(PS_ERR_INVALID, "ps_muon_update: parameters must be FP32, BF16 or FP16");
  if (upd_dtype != PS_F32 && upd_dtype != PS_BF16 && upd_dtype != PS_F16)
    return fail(PS_ERR_INVALID, "ps_muon_update: updates must be FP32, BF16 or FP16");
  if (!std::isfinite(decay) || !std::isfinite(alpha))
    return fail(PS_ERR_INVALID, "ps_muon_update: factors must be finite");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PS_F32:
      return muon_update_in<float>(upd_dtype, params, count, elems, decay, alpha, updates, st->sms, s);
    case PS_BF16:
      return muon_update_in<__nv_bfloat16>(upd_dtype, params, count, elems, decay, alpha, updates, st->sms, s);
    default:
      return muon_update_in<__half>(upd_dtype, params, count, elems, decay, alpha, updates, st->sms, s);
  }
}

int ps_update_stats(const void* x, int x_dtype, int64_t L, int64_t elems, int64_t* nan_count,
                    int64_t* inf_count, float* max_abs, void* stream) {
  if (!x || !nan_count || !inf_count || !max_abs) return fail(PS_ERR_INVALID, "ps_update_stats: null pointer");
  if (L < 1 || elems < 1) return fail(PS_ERR_INVALID, "ps_update_stats: empty input");
  if (x_dtype != PS_F16 && x_dtype != PS_BF16 && x_dtype != PS_F32)
    return fail(PS_ERR_INVALID, "ps_update_stats: updates must be FP16, BF16 or FP32");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (x_dtype) {
    case PS_F16:
      return launch_update_stats<__half>(x, L, elems, nan_count, inf_count, max_abs, st->sms, s);
    case PS_BF16:
      return launch_update_stats<__nv_bfloat16>(x, L, elems, nan_count, inf_count, max_abs, st->sms, s);
    default:
      return launch_update_stats<float>(x, L, elems, nan_count, inf_count, max_abs, st->sms, s);
  }
}

int ps_gram(const void* x, void* out, int64_t L, int64_t rows, int64_t cols, int64_t x_ld,
            void* stream) {
  return gram_impl(x, out, L, rows, cols, x_ld, rows > cols, static_cast<cudaStream_t>(stream));
}

int ps_square(const void* a, const void* c, void* out, int64_t L, int64_t n, float alpha,
              float beta, float diag, void* stream) {
  return sym_product_impl(a, a, c, out, L, n, alpha, beta, diag,
                          static_cast<cudaStream_t>(stream), "ps_square");
}

int ps_sym_product(const void* p, const void* q, const void* c, void* out, int64_t L, int64_t n,
                   float alpha, float beta, float diag, void* stream) {
  return sym_product_impl(p, q, c, out, L, n, alpha, beta, diag,
                          static_cast<cudaStream_t>(stream), "ps_sym_product");
}

int ps_apply(const void* b, const void* x, void* y, int64_t L, int64_t rows, int64_t cols,
             int64_t x_ld, float residual, int y_dtype, int64_t y_ld, void* stream) {
  return apply_impl(b, x, y, L, rows, cols, x_ld, residual, y_dtype, y_ld, rows > cols,
                    static_cast<cudaStream_t>(stream));
}

int ps_add_diag(const void* in, void* out, int64_t L, int64_t n, float a, void* stream) {
  return add_diag_impl(in, out, L, n, a, static_cast<cudaStream_t>(stream));
}

int64_t ps_circuit_workspace_bytes(int64_t L, int64_t rows, int64_t cols, int buffers) {
  ps_problem p;
  std::memset(&p, 0, sizeof(p));
  p.L = L;
  p.rows = rows;
  p.cols = cols;
  return ps_circuit_grouped_workspace_bytes(&p, 1, buffers);
}

int ps_circuit(const void* x, int x_dtype, int64_t L, int64_t rows, int64_t cols, int64_t sL,
               int64_t sR, int64_t sC, void* y, int y_dtype, int n_outer,
               const float* residuals, const int32_t* n_steps, const ps_step* steps, int buffers,
               float eps, void* workspace, int64_t workspace_bytes, void* stream) {
  ps_problem p;
  p.x = x;
  p.x_dtype = x_dtype;
  p.L = L;
  p.rows = rows;
  p.cols = cols;
  p.sL = sL;
  p.sR = sR;
  p.sC = sC;
  p.y = y;
  p.y_dtype = y_dtype;
  return ps_circuit_grouped(&p, 1, n_outer, residuals, n_steps, steps, buffers, eps, workspace,
                            workspace_bytes, stream);
}

int64_t ps_circuit_grouped_workspace_bytes(const ps_problem* probs, int n_probs, int buffers) {
  DeviceState* st = nullptr;
  if (device_state(&st)) return -1;
  GroupedPlan plan;
  if (make_grouped_plan(probs, n_probs, buffers, st->sms, &plan)) return -1;
  return plan.total;
}

int ps_circuit_grouped(const ps_problem* probs, int n_probs, int n_outer, const float* residuals,
                       const int32_t* n_steps, const ps_step* steps, int buffers, float eps,
                       void* workspace, int64_t workspace_bytes, void* stream) {
  return ps_circuit_grouped_update(probs, nullptr, n_probs, n_outer, residuals, n_steps, steps,
                                   buffers, eps, workspace, workspace_bytes, stream);
}

static int circuit_grouped_impl(const ps_problem* probs, const ps_update* updates, int n_probs,
                                int n_outer, const float* residuals, const int32_t* n_steps,
                                const ps_step* steps, int buffers, float eps, void* workspace,
                                int64_t workspace_bytes, void* stream, const CircuitPush* push);

int ps_circuit_grouped_update(const ps_problem* probs, const ps_update* updates, int n_probs,
                              int n_outer, const float* residuals, const int32_t* n_steps,
                              const ps_step* steps, int buffers, float eps, void* workspace,
                              int64_t workspace_bytes, void* stream) {
  return circuit_grouped_impl(probs, updates, n_probs, n_outer, residuals, n_steps, steps, buffers,
                              eps, workspace, workspace_bytes, stream, nullptr);
}

int ps_circuit_grouped_push(const ps_problem* probs, int n_probs, int n_outer, const float* residuals,
                            const int32_t* n_steps, const ps_step* steps, int buffers, float eps,
                            void* workspace, int64_t workspace_bytes, const void* local_base,
                            const void* const* peer_bases, int n_peers, int n_phases,
                            const int32_t* phase_ends, void* stream) {
  if (n_peers < 0 || n_peers > ps::circ::MAX_PEERS)
    return fail(PS_ERR_INVALID, "ps_circuit_grouped_push: n_peers must be in [0, %d]",
                ps::circ::MAX_PEERS);
  if (n_peers > 0 && (!local_base || !peer_bases))
    return fail(PS_ERR_INVALID, "ps_circuit_grouped_push: null local_base or peer_bases");
  for (int k = 0; k < n_peers; ++k)
    if (!peer_bases[k] || !aligned16(peer_bases[k]))
      return fail(PS_ERR_INVALID, "ps_circuit_grouped_push: peer base %d is null or misaligned", k);
  if (n_phases < 1 || n_phases > ps::circ::MAX_PHASES)
    return fail(PS_ERR_INVALID, "ps_circuit_grouped_push: n_phases must be in [1, %d]",
                ps::circ::MAX_PHASES);
  if (!probs || n_probs <= 0) return fail(PS_ERR_INVALID, "ps_circuit: bad problem list");
  if (n_phases > 1) {
    if (!phase_ends) return fail(PS_ERR_INVALID, "ps_circuit_grouped_push: null phase_ends");
    for (int i = 0; i < n_probs; ++i) {
      int32_t prev = 0;
      for (int k = 0; k < n_phases; ++k) {
        const int32_t e = phase_ends[i * n_phases + k];
        if (e < prev || (k == n_phases - 1 && e != probs[i].L))
          return fail(PS_ERR_INVALID,
                      "ps_circuit_grouped_push: phase_ends of problem %d must be non-decreasing "
                      "and end at its L", i);
        prev = e;
      }
    }
  }
  CircuitPush push;
  push.local_base = static_cast<const uint8_t*>(local_base);
  push.peer_bases = peer_bases;
  push.n_peers = n_peers;
  push.n_phases = n_phases;
  push.phase_ends = n_phases > 1 ? phase_ends : nullptr;
  return circuit_grouped_impl(probs, nullptr, n_probs, n_outer, residuals, n_steps, steps, buffers,
                              eps, workspace, workspace_bytes, stream, &push);
}

int ps_circuit_grouped_signal(const ps_problem* probs, int n_probs, int n_outer,
                              const float* residuals, const int32_t* n_steps, const ps_step* steps,
                              int buffers, float eps, void* workspace, int64_t workspace_bytes,
                              int n_phases, const int32_t* phase_ends, unsigned* signals,
                              void* stream) {
  if (!signals || !aligned16(signals))
    return fail(PS_ERR_INVALID, "ps_circuit_grouped_signal: signals must be 16-byte aligned device memory");
  if (n_phases < 1 || n_phases > ps::circ::MAX_PHASES)
    return fail(PS_ERR_INVALID, "ps_circuit_grouped_signal: n_phases must be in [1, %d]",
                ps::circ::MAX_PHASES);
  if (!probs || n_probs <= 0) return fail(PS_ERR_INVALID, "ps_circuit: bad problem list");
  if (n_phases > 1) {
    if (!phase_ends) return fail(PS_ERR_INVALID, "ps_circuit_grouped_signal: null phase_ends");
    for (int i = 0; i < n_probs; ++i) {
      int32_t prev = 0;
      for (int k = 0; k < n_phases; ++k) {
        const int32_t e = phase_ends[i * n_phases + k];
        if (e < prev || (k == n_phases - 1 && e != probs[i].L))
          return fail(PS_ERR_INVALID,
                      "ps_circuit_grouped_signal: phase_ends of problem %d must be non-decreasing "
                      "and end at its L", i);
        prev = e;
      }
    }
  }
  CircuitPush push;
  push.n_phases = n_phases;
  push.phase_ends = n_phases > 1 ? phase_ends : nullptr;
  push.sig = signals;
  return circuit_grouped_impl(probs, nullptr, n_probs, n_outer, residuals, n_steps, steps, buffers,
                              eps, workspace, workspace_bytes, stream, &push);
}

int ps_stream_wait_flag(void* stream, const unsigned* flag, unsigned value) {
  static PFN_cuStreamWaitValue32_v11070 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuStreamWaitValue32", &p, 11070, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuStreamWaitValue32_v11070>(p);
  });
  if (!flag || reinterpret_cast<uintptr_t>(flag) % 4)
    return fail(PS_ERR_INVALID, "ps_stream_wait_flag: flag must be a 4-byte aligned device address");
  if (!fn) return fail(PS_ERR_CUDA, "cuStreamWaitValue32 entry point unavailable");
  CUresult r = fn(static_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(flag), value,
                  CU_STREAM_WAIT_VALUE_GEQ);
  if (r != CUDA_SUCCESS) return fail(PS_ERR_CUDA, "cuStreamWaitValue32 failed (%d)", static_cast<int>(r));
  return PS_OK;
}

static int circuit_grouped_impl(const ps_problem* probs, const ps_update* updates, int n_probs,
                                int n_outer, const float* residuals, const int32_t* n_steps,
                                const ps_step* steps, int buffers, float eps, void* workspace,
                                int64_t workspace_bytes, void* stream, const CircuitPush* push) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!workspace) return fail(PS_ERR_INVALID, "ps_circuit: null workspace");
  if (!probs || n_probs <= 0) return fail(PS_ERR_INVALID, "ps_circuit: bad problem list");
  int rc = validate_table(n_outer, residuals, n_steps, steps, buffers);
  if (rc) return rc;
  for (int i = 0; i < n_probs; ++i) {
    const bool upd = updates && updates[i].p;
    if (!probs[i].x || (!probs[i].y && !upd))
      return fail(PS_ERR_INVALID, "ps_circuit: problem %d has a null pointer", i);
    if (upd) {
      const ps_update& u = updates[i];
      const ps_problem& q = probs[i];
      if (u.p_dtype != PS_F32 && u.p_dtype != PS_BF16 && u.p_dtype != PS_F16)
        return fail(PS_ERR_INVALID, "ps_circuit: update %d: parameters must be FP32, BF16 or FP16", i);
      if (!std::isfinite(u.decay) || !std::isfinite(u.alpha))
        return fail(PS_ERR_INVALID, "ps_circuit: update %d: factors must be finite", i);
      if (q.y_dtype != PS_F16 && q.y_dtype != PS_F32 && q.y_dtype != PS_BF16)
        return fail(PS_ERR_INVALID, "ps_circuit: update %d: y_dtype must be FP16, FP32 or BF16", i);
      if (q.rows % 8 || q.cols % 8 || !aligned16(u.p) || (q.cols * elem_bytes(u.p_dtype)) % 16 ||
          !use_pair(false, std::min(q.rows, q.cols)))
        return fail(PS_ERR_UNSUPPORTED,
                    "ps_circuit: update %d needs the CTA-pair kernel, rows and cols multiples of 8 "
                    "and a 16-byte aligned bank with 16-byte rows", i);
    }
  }
  DeviceState* st = nullptr;
  if ((rc = device_state(&st))) return rc;
  GroupedPlan plan;
  if ((rc = make_grouped_plan(probs, n_probs, buffers, st->sms, &plan))) return rc;
  if (workspace_bytes < plan.total) return fail(PS_ERR_WORKSPACE, "ps_circuit: workspace too small");
  if (!aligned16(workspace)) return fail(PS_ERR_INVALID, "ps_circuit: workspace misaligned");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int np = n_probs;

  auto buf_ptr = [&](int prob, int b) -> void* {
    const GroupedPlan::Prob& p = plan.probs[prob];
    const GroupedPlan::NGroup& g = plan.groups[p.group];
    return ws + g.buf_off + b * g.buf_bytes + p.goff * p.lay.n * p.lay.n * 2;
  };
  std::vector<int> cur(np, 0);
  std::vector<bool> direct(np);
  // Square buffers live only inside this call, so they are kept as
  // upper-triangle blocks (no mirrored stores).
  const bool tri = true;
  std::vector<NormJob> norm_jobs(np);
  for (int i = 0; i < np; ++i) {
    const ps_problem& q = probs[i];
    const GroupedPlan::Prob& p = plan.probs[i];
    norm_jobs[i] = {q.x, q.x_dtype, q.L, q.rows, q.cols, q.sL, q.sR, q.sC, ws + p.xh_off[0],
                    p.lay.Rp, p.lay.Cp, reinterpret_cast<double*>(ws + p.norm_off),
                    reinterpret_cast<unsigned*>(ws + p.cnt_off)};
  }
  if (push) {
    // Checked before anything is launched, so a caller can take another path.
    if (!use_circuit_kernel(plan, np, n_outer, n_steps, buffers))
      return fail(PS_ERR_UNSUPPORTED,
                  "ps_circuit_grouped_push/_signal: the problems do not fit one whole-circuit launch");
    for (int i = 0; i < np; ++i) {
      const ps_problem& q = probs[i];
      const GroupedPlan::Prob& p = plan.probs[i];
      if (!((q.y_dtype == PS_F16 || q.y_dtype == PS_F32 || q.y_dtype == PS_BF16) &&
            p.lay.Rp == q.rows && p.lay.Cp == q.cols && (q.cols * elem_bytes(q.y_dtype)) % 16 == 0 &&
            aligned16(q.y)))
        return fail(PS_ERR_UNSUPPORTED,
                    "ps_circuit_grouped_push/_signal: problem %d needs rows and cols multiples of 8 and a "
                    "16-byte aligned y with 16-byte rows", i);
      if (push->n_peers > 0 && static_cast<const uint8_t*>(q.y) < push->local_base)
        return fail(PS_ERR_INVALID, "ps_circuit_grouped_push: y of problem %d lies before local_base", i);
    }
  }
  std::vector<unsigned> chain_base(plan.groups.size(), 0u);
  {
    // chain and fused-normalisation counters start at zero in every call
    cudaError_t e = cudaMemsetAsync(ws + plan.ctr_off, 0, plan.ctr_bytes, s);
    if (e != cudaSuccess) return cuda_fail(e, "counters memset");
  }
  // The normalisations of all problems, batched by input type.
  if ((rc = normalize_jobs(norm_jobs, eps, st->sms, s))) return rc;
  for (int i = 0; i < np; ++i) {
    const ps_problem& q = probs[i];
    const GroupedPlan::Prob& p = plan.probs[i];
    // The last apply writes straight into y when y's layout allows TMA stores
    // (or applies the update straight into the bank, checked above).
    direct[i] = (updates && updates[i].p) ||
                ((q.y_dtype == PS_F16 || q.y_dtype == PS_F32 || q.y_dtype == PS_BF16) &&
                 p.lay.Rp == q.rows && p.lay.Cp == q.cols &&
                 (q.cols * elem_bytes(q.y_dtype)) % 16 == 0 && aligned16(q.y));
  }
  // Chain launches count completed tiles per matrix from zero within this call.
  if (use_circuit_kernel(plan, np, n_outer, n_steps, buffers)) {
    // every stage of every problem in one persistent launch
    if ((rc = circuit_kernel_run(plan, probs, updates, np, n_outer, residuals, n_steps, steps, buffers,
                                 ws, direct, s, push)))
      return rc;
    for (int i = 0; i < np; ++i) {
      if (direct[i]) continue;
      const GroupedPlan::Prob& p = plan.probs[i];
      const ps_problem& q = probs[i];
      // the final apply wrote Xh[1 - cur], cur flipping after each of the other applies
      const int fin = (n_outer - 1) & 1 ? 0 : 1;
      if ((rc = copy_out(ws + p.xh_off[fin], p.lay.Rp, p.lay.Cp, q.rows, q.cols, q.L, q.y,
                         q.y_dtype, st->sms, s)))
        return rc;
    }
    return PS_OK;
  }
  int off = 0;
  for (int t = 0; t < n_outer; ++t) {
    // The Grams of all problems, batched into one launch per kernel variant.
    {
      JobSink sink;
      for (int i = 0; i < np; ++i) {
        const GroupedPlan::Prob& p = plan.probs[i];
        if ((rc = gram_impl(ws + p.xh_off[cur[i]], buf_ptr(i, 0), probs[i].L, p.lay.Rp, p.lay.Cp,
                            p.lay.Cp, p.lay.tall, s, tri)))
          return rc;
      }
      if ((rc = sink.flush(s))) return rc;
    }
    const int last = steps[off + n_steps[t] - 1].dst;
    for (size_t gi = 0; gi < plan.groups.size(); ++gi) {
      const GroupedPlan::NGroup& g = plan.groups[gi];
      uint8_t* base = ws + g.buf_off;
      if (use_chain(g.n, buffers)) {
        // All inner iterations of this outer iteration in chain launches of
        // up to MAX_STEPS steps each.
        unsigned* done = reinterpret_cast<unsigned*>(ws + g.ctr_off);
        const unsigned per_step =
            static_cast<unsigned>(ps::chain::SIGNALS_PER_TILE * pair_sym_tiles(g.n));
        for (int k0 = 0; k0 < n_steps[t]; k0 += ps::chain::MAX_STEPS) {
          const int S = std::min(n_steps[t] - k0, ps::chain::MAX_STEPS);
          if ((rc = chain_launch(base, g.buf_bytes, buffers, g.Ltot, g.n, steps + off + k0, S, done,
                                 chain_base[gi], s)))
            return rc;
          chain_base[gi] += static_cast<unsigned>(S) * per_step;
        }
        continue;
      }
      // One launch per inner iteration covers every problem with this n.
      for (int k = 0; k < n_steps[t]; ++k) {
        const ps_step& q = steps[off + k];
        if ((rc = sym_product_impl(base + q.src * g.buf_bytes, base + q.src * g.buf_bytes,
                                   base + q.add * g.buf_bytes, base + q.dst * g.buf_bytes, g.Ltot,
                                   g.n, q.alpha, q.beta, q.diag, s, "ps_circuit(square)", tri)))
          return rc;
      }
    }
    off += n_steps[t];
    const bool final_iter = t == n_outer - 1;
    // The applies of all problems, batched likewise.
    JobSink sink;
    for (int i = 0; i < np; ++i) {
      const GroupedPlan::Prob& p = plan.probs[i];
      const ps_problem& q = probs[i];
      const int64_t Rp = p.lay.Rp, Cp = p.lay.Cp;
      if (final_iter && direct[i]) {
        const bool upd = updates && updates[i].p;
        rc = apply_impl(buf_ptr(i, last), ws + p.xh_off[cur[i]], upd ? updates[i].p : q.y, q.L, Rp,
                        Cp, Cp, residuals[t], q.y_dtype, q.cols, p.lay.tall, s, tri,
                        upd ? &updates[i] : nullptr);
      } else {
        rc = apply_impl(buf_ptr(i, last), ws + p.xh_off[cur[i]], ws + p.xh_off[1 - cur[i]], q.L,
                        Rp, Cp, Cp, residuals[t], PS_F16, Cp, p.lay.tall, s, tri);
        cur[i] = 1 - cur[i];
      }
      if (rc) return rc;
    }
    if ((rc = sink.flush(s))) return rc;
  }
  for (int i = 0; i < np; ++i) {
    if (direct[i]) continue;
    const GroupedPlan::Prob& p = plan.probs[i];
    const ps_problem& q = probs[i];
    if ((rc = copy_out(ws + p.xh_off[cur[i]], p.lay.Rp, p.lay.Cp, q.rows, q.cols, q.L, q.y,
                       q.y_dtype, st->sms, s)))
      return rc;
  }
  return PS_OK;
}

// ---------------------------------------------------------------- Gram Newton-Schulz
// The recurrence of polar_switch/gram_newton_schulz.py:75-122 as one C call:
// R = X X^T (X^T X for tall X) once, per iteration Z = c R R + b R, Q = Z + a I
// after a (re)start else Q = Q Z + a Q, and between restarts R = Z (R Z + a R)
// + a (R Z + a R); at a restart X <- Q X and R is formed again; finally
// X <- Q X. The buffers are stored in full (mirrored): a product of two
// different matrices is symmetric only up to rounding, so unlike a square its
// diagonal blocks are not bit-symmetric and could not be read back transposed
// exactly; full storage keeps every step identical to the op-by-op recurrence.
constexpr int kGnsBuffers = 5;

int64_t ps_gns_workspace_bytes(int64_t L, int64_t rows, int64_t cols) {
  if (!dims_ok(L, rows, cols)) return fail(PS_ERR_INVALID, "ps_gns: bad sizes");
  DeviceState* st = nullptr;
  if (device_state(&st)) return -1;
  return circuit_layout(L, rows, cols, kGnsBuffers, st->sms).total;
}

int ps_gns(const void* x, int x_dtype, int64_t L, int64_t rows, int64_t cols, int64_t sL,
           int64_t sR, int64_t sC, void* y, int y_dtype, int n_iter, const float* coeffs,
           int n_resets, const int32_t* resets, float eps, void* workspace, int64_t workspace_bytes,
           void* stream) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!x || !y || !workspace || !coeffs || (n_resets > 0 && !resets))
    return fail(PS_ERR_INVALID, "ps_gns: null pointer");
  if (!dims_ok(L, rows, cols)) return fail(PS_ERR_INVALID, "ps_gns: bad sizes");
  if (rows == cols)
    return fail(PS_ERR_INVALID, "ps_gns: square matrices take Polar Express, not the Gram recurrence");
  if (n_iter < 1 || n_iter > 64 || n_resets < 0 || n_resets > 64)
    return fail(PS_ERR_INVALID, "ps_gns: bad iteration or restart count");
  for (int i = 0; i < 3 * n_iter; ++i)
    if (!std::isfinite(coeffs[i])) return fail(PS_ERR_INVALID, "ps_gns: non-finite coefficient");
  if (elem_bytes(x_dtype) == 0 || elem_bytes(y_dtype) == 0)
    return fail(PS_ERR_INVALID, "ps_gns: bad dtype");
  if (!aligned16(workspace)) return fail(PS_ERR_INVALID, "ps_gns: workspace misaligned");
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  const CircuitLayout lay = circuit_layout(L, rows, cols, kGnsBuffers, st->sms);
  if (workspace_bytes < lay.total) return fail(PS_ERR_WORKSPACE, "ps_gns: workspace too small");
  auto is_reset = [&](int i) {
    for (int k = 0; k < n_resets; ++k)
      if (resets[k] == i) return true;
    return false;
  };
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint8_t* xh[2] = {ws, ws + lay.xh_bytes};
  auto buf = [&](int k) -> void* { return ws + 2 * lay.xh_bytes + k * lay.buf_bytes; };
  uint8_t* norm = ws + 2 * lay.xh_bytes + kGnsBuffers * lay.buf_bytes;
  const int64_t Rp = lay.Rp, Cp = lay.Cp, n = lay.n;
  const bool tall = lay.tall, tri = false;
  int R = 0, Z = 1, Q = 2, Q2 = 3, RZ = 4, cur = 0;
  if ((rc = normalize_impl(x, x_dtype, L, rows, cols, sL, sR, sC, eps, xh[0], Rp, Cp, norm,
                           lay.norm_bytes, s)))
    return rc;
  if ((rc = gram_impl(xh[cur], buf(R), L, Rp, Cp, Cp, tall, s, tri))) return rc;
  const int last = n_iter - 1;
  for (int i = 0; i < n_iter; ++i) {
    const float a = coeffs[3 * i], b = coeffs[3 * i + 1], c = coeffs[3 * i + 2];
    const bool restart = i != 0 && is_reset(i);
    if (restart) {
      if ((rc = apply_impl(buf(Q), xh[cur], xh[1 - cur], L, Rp, Cp, Cp, 0.f, PS_F16, Cp, tall, s,
                           tri)))
        return rc;
      cur = 1 - cur;
      if ((rc = gram_impl(xh[cur], buf(R), L, Rp, Cp, Cp, tall, s, tri))) return rc;
    }
    if ((rc = sym_product_impl(buf(R), buf(R), buf(R), buf(Z), L, n, c, b, 0.f, s, "ps_gns", tri)))
      return rc;
    if (i == 0 || is_reset(i)) {
      if ((rc = add_diag_impl(buf(Z), buf(Q), L, n, a, s))) return rc;
    } else {
      if ((rc = sym_product_impl(buf(Q), buf(Z), buf(Q), buf(Q2), L, n, 1.f, a, 0.f, s, "ps_gns",
                                 tri)))
        return rc;
      std::swap(Q, Q2);
    }
    if (i < last && !is_reset(i + 1)) {
      if ((rc = sym_product_impl(buf(R), buf(Z), buf(R), buf(RZ), L, n, 1.f, a, 0.f, s, "ps_gns",
                                 tri)))
        return rc;
      if ((rc = sym_product_impl(buf(Z), buf(RZ), buf(RZ), buf(R), L, n, 1.f, a, 0.f, s, "ps_gns",
                                 tri)))
        return rc;
    }
  }
  // X <- Q X, straight into y when its layout allows TMA stores.
  const bool direct = (y_dtype == PS_F16 || y_dtype == PS_F32 || y_dtype == PS_BF16) &&
                      Rp == rows && Cp == cols && (cols * elem_bytes(y_dtype)) % 16 == 0 &&
                      aligned16(y);
  if (direct)
    return apply_impl(buf(Q), xh[cur], y, L, Rp, Cp, Cp, 0.f, y_dtype, cols, tall, s, tri);
  if ((rc = apply_impl(buf(Q), xh[cur], xh[1 - cur], L, Rp, Cp, Cp, 0.f, PS_F16, Cp, tall, s, tri)))
    return rc;
  return copy_out(xh[1 - cur], Rp, Cp, rows, cols, L, y, y_dtype, st->sms, s);
}

// ---------------------------------------------------------------- no-alloc normalise
// Device address of ps::g_noalloc_partials per device. Host code may not pass
// the array's name to a kernel: on the host it is a stand-in symbol, not a
// device address. The address is looked up once per device, with that device
// current, on the first ps_normalize_noalloc call there.
static std::mutex g_noalloc_mu;
static double* g_noalloc_ptr[kMaxDevices] = {};

static int noalloc_scratch(double** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(PS_ERR_UNSUPPORTED, "device index %d", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, ps::g_noalloc_partials);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(noalloc scratch)");
    g_noalloc_ptr[dev] = static_cast<double*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return PS_OK;
}

int ps_normalize_noalloc(const void* x, int x_dtype, int64_t L, int64_t rows, int64_t cols,
                         int64_t sL, int64_t sR, int64_t sC, float eps, void* xh, int64_t rows_p,
                         int64_t cols_p, void* stream) {
  if (!x || !xh) return fail(PS_ERR_INVALID, "ps_normalize_noalloc: null pointer");
  if (!dims_ok(L, rows, cols) || rows_p < rows || cols_p < cols)
    return fail(PS_ERR_INVALID, "ps_normalize_noalloc: bad sizes");
  if (elem_bytes(x_dtype) == 0) return fail(PS_ERR_INVALID, "ps_normalize_noalloc: bad dtype");
  if (!(eps > 0.f)) return fail(PS_ERR_INVALID, "ps_normalize_noalloc: eps must be positive");
  if (L > PS_NORMALIZE_NOALLOC_MAX_PARTIALS)
    return fail(PS_ERR_UNSUPPORTED,
                "ps_normalize_noalloc: L=%lld matrices exceed the built-in scratch of %d partial "
                "sums; use ps_normalize with a caller workspace",
                (long long)L, PS_NORMALIZE_NOALLOC_MAX_PARTIALS);
  DeviceState* st = nullptr;
  int rc = device_state(&st);
  if (rc) return rc;
  double* partial = nullptr;
  if ((rc = noalloc_scratch(&partial))) return rc;
  // Same chunking as ps_normalize whenever it fits, so both entry points give
  // identical results; otherwise fewer chunks per matrix.
  int chunks = norm_chunks(L, rows, cols, st->sms);
  if (L * chunks > PS_NORMALIZE_NOALLOC_MAX_PARTIALS)
    chunks = static_cast<int>(PS_NORMALIZE_NOALLOC_MAX_PARTIALS / L);
  int64_t ce = ps::norm_chunk_elems(rows * cols);
  const int64_t max_per = PS_NORMALIZE_NOALLOC_MAX_PARTIALS / L;
  if ((rows * cols + ce - 1) / ce > max_per)
    ce = round_up((rows * cols + max_per - 1) / max_per, ps::NORM_CHUNK);
  // Pass 1 writes every one of the L * chunks partial sums before pass 2 reads
  // them, so nothing left in the scratch by an earlier call is ever read.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (x_dtype) {
    case PS_F16:
      return launch_normalize<__half>(x, L, rows, cols, sL, sR, sC, eps, xh, rows_p, cols_p,
                                      partial, chunks, ce, st->sms, s);
    case PS_BF16:
      return launch_normalize<__nv_bfloat16>(x, L, rows, cols, sL, sR, sC, eps, xh, rows_p,
                                             cols_p, partial, chunks, ce, st->sms, s);
    case PS_F32:
      return launch_normalize<float>(x, L, rows, cols, sL, sR, sC, eps, xh, rows_p, cols_p,
                                     partial, chunks, ce, st->sms, s);
    default:
      return launch_normalize<double>(x, L, rows, cols, sL, sR, sC, eps, xh, rows_p, cols_p,
                                      partial, chunks, ce, st->sms, s);
  }
}

}  // extern "C"
