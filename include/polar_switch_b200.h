/*
 * polar_switch_b200 -- C ABI of the B200 (sm_100a) Polar Switch orthogonalizer.
 *
 * Every entry point takes plain device pointers, sizes, FP32 scalars and a
 * cudaStream_t passed as `void*` (NULL = legacy default stream). All work is
 * enqueued on that stream; no entry point synchronises the host except
 * ps_get_status(). The library allocates no device memory: the caller owns
 * every buffer, including the scratch `workspace` of ps_normalize/ps_circuit.
 *
 * Return value: PS_OK (0) or a negative PS_ERR_* code; ps_last_error()
 * returns a message for the calling thread's last failure.
 *
 * Device state: per device, the first call looks up the device addresses of
 * the library's module variables (the status word, the ps_normalize_noalloc
 * scratch) and caches them for the life of the process. The library does not
 * survive a cudaDeviceReset() or a destroyed and recreated primary context on
 * a device it has already used: those cached addresses go stale.
 *
 * FP16 matrices passed to gram/square/sym_product/apply are row-major with a
 * row pitch (`*_ld`, in elements) that is a multiple of 8, on 16-byte aligned
 * addresses; batch `l` starts at `ptr + l * rows * ld`.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   polar_switch/__init__.py:25-45          _run                -> ps_circuit
 *   polar_switch/__init__.py:34-35          FP32 normalise      -> ps_normalize
 *   polar_switch/gemm_symmetric_fused.py:291-293 / triton_kernels.py:72-74
 *                                           gram(X, tall, out)  -> ps_gram
 *   polar_switch/gemm_symmetric_fused.py:296-301 / triton_kernels.py:77-79
 *                                           square(A, C, out, alpha, beta, diag) -> ps_square
 *   polar_switch/gram_newton_schulz.py:64-72 sym_baddbmm(A, B, C, alpha, beta)   -> ps_sym_product
 *   polar_switch/gemm_symmetric_fused.py:304-309 / triton_kernels.py:82-87
 *                                           apply(X, B, tall, residual) -> ps_apply
 *   polar_switch/gram_newton_schulz.py:107  Q = Z + a*I          -> ps_add_diag
 *   polar_switch/gram_newton_schulz.py:75-122 rectangular GNS     -> ps_gns
 *   training/muon.py:59-86 (buckets of one step) -> ps_circuit_grouped
 *   training/muon.py:63-74 momentum/Nesterov/stack/cast -> ps_muon_direction
 *   training/muon.py:84-86 decay and scaled update     -> ps_muon_update
 *   training/diagnostics.py:161-165 NaN / inf counts, max |x| -> ps_update_stats
 *   (no single counterpart) split-matrix pieces -> ps_sumsq, ps_scale_cast, ps_gram_f32
 */
#ifndef POLAR_SWITCH_B200_H
#define POLAR_SWITCH_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define PS_API __attribute__((visibility("default")))
#else
#define PS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define PS_OK 0
#define PS_ERR_INVALID (-1)     /* bad argument (null pointer, size, alignment, table) */
#define PS_ERR_CUDA (-2)        /* a CUDA runtime/driver call failed */
#define PS_ERR_UNSUPPORTED (-3) /* device or shape outside what the kernels support */
#define PS_ERR_WORKSPACE (-4)   /* workspace smaller than ps_*_workspace_bytes() */

/* dtype codes */
#define PS_F16 0
#define PS_F32 1
#define PS_BF16 2
#define PS_F64 3


/* One inner iteration (w, i, r, a, b, c) of a coefficient table:
 * B[dst] = alpha * B[src] @ B[src] + beta * B[add] + diag * I
 * (polar_switch/coefficients.py:1-8). */
typedef struct ps_step {
  int32_t dst, src, add;
  float alpha, beta, diag;
} ps_step;

/* Library version (major * 10000 + minor * 100 + patch). */
PS_API int ps_version(void);

/* Message describing the calling thread's last error ("" if none). */
PS_API const char* ps_last_error(void);

/* Device status word of the current device: 0, or the code of the first
 * bounded wait inside a kernel that ran out (the kernel then returned early
 * and its output is undefined). Synchronous; `clear` resets it to 0. */
PS_API int ps_get_status(int* status, int clear);

/* Upper bound, in SM clock cycles, for every spin-wait inside the kernels
 * launched afterwards by this process (default 2^32, about two seconds). */
PS_API int ps_set_wait_limit(long long cycles);

/* Launches one kernel whose single wait can never be satisfied, so that it
 * runs out after `limit_cycles` and records its status code (5). Used by the
 * tests of the bounded-wait path. */
PS_API int ps_selftest_wait(long long limit_cycles, void* stream);

/* Launches one chain kernel (see ps_set_chain) whose second inner iteration
 * waits for a completion count that never arrives: those waits run out after
 * `limit_cycles` and record status code 6 (dependency timeout), and the
 * kernel returns early. `workspace`: at least PS_SELFTEST_CHAIN_WORKSPACE_BYTES
 * of device memory, 16-byte aligned (overwritten). limit_cycles must be at
 * most a quarter of the ps_set_wait_limit value. Used by the tests of the
 * bounded-wait path of the chain kernel. */
#define PS_SELFTEST_CHAIN_WORKSPACE_BYTES (1 << 20)
PS_API int ps_selftest_chain_wait(void* workspace, int64_t workspace_bytes, long long limit_cycles,
                                  void* stream);

/* Number of kernels this library has launched in the process so far. */
PS_API long long ps_launch_count(void);

/* Profiling of the library's own launches: enable=1 clears the records and
 * brackets every later launch with CUDA events on its stream; enable=0 stops
 * recording. ps_profile_read waits for the recorded launches of one class
 * (0 normalise, 1 gram, 2 square/symmetric product, 3 apply, 4 other,
 * 5 whole circuit in one launch) and
 * returns their summed device time, count, algorithmic FLOPs and algorithmic
 * HBM bytes. */
PS_API int ps_profile_enable(int enable);
PS_API int ps_profile_read(int kind, double* total_ms, int64_t* launches, double* flops,
                           double* bytes);

/* Selects the GEMM kernel for later launches: 0 = one-CTA kernel (128 x 256
 * tiles), 1 (default) = CTA-pair kernel (tcgen05 cta_group::2, 256 x 256
 * tiles over two SMs) for every product, 2 = CTA pairs for squares of buffers
 * with n <= 1024 and the one-CTA kernel for everything else. All compute the
 * same products with the same rounding. Returns the previous mode
 * (PS_ERR_INVALID for other values). */
PS_API int ps_set_cta_pairs(int mode);

/* How the inner iterations of ps_circuit / ps_circuit_grouped run on the
 * CTA-pair path (every n under ps_set_cta_pairs(1)): 1 (default) = one persistent
 * launch per outer iteration for all of them ("chain": a step of a matrix
 * starts as soon as that matrix's previous step is stored, so its buffers are
 * reused from L2), 0 = one launch per inner iteration. Same bits either way.
 * Returns the previous mode (PS_ERR_INVALID for other values). No counterpart
 * in the reference (its inner loop, polar_switch/__init__.py:42-43, issues one
 * kernel per inner iteration). */
PS_API int ps_set_chain(int mode);

/* How ps_circuit / ps_circuit_grouped run on the CTA-pair path: 1 (default) =
 * one persistent launch for every stage of every problem (each matrix's Gram,
 * inner iterations and apply chained through per-matrix completion counters,
 * bounded waits), 0 = one launch per stage. Same bits either way;
 * up to 8 problems, 3 buffers and 48 stages (else per-stage launches).
 * Returns the previous mode (PS_ERR_INVALID for other values). Replaces the
 * whole loop of polar_switch/__init__.py:40-44 with one launch. */
PS_API int ps_set_circuit_kernel(int mode);

/* How ps_circuit / ps_circuit_grouped normalise contiguous, unpadded inputs:
 * 1 = one read of the input (a persistent kernel keeps each chunk in shared
 * memory until its matrix's norm is known), 0 (default) = two passes over the
 * input (sums of squares, then scale and cast). Same bits either way; the
 * single read measured slower than the two passes at the Qwen step. Returns
 * the previous mode (PS_ERR_INVALID for other values). No counterpart in the
 * reference (polar_switch/__init__.py:34-35 normalises in two torch ops). */
PS_API int ps_set_fused_normalize(int mode);

/* Caps the number of CTAs (one per SM) of the persistent GEMM grids launched
 * afterwards; 0 (default) = every SM. Leaving SMs free lets a collective on
 * another stream run beside the GEMMs. Returns the previous cap. */
PS_API int ps_set_max_ctas(int max_ctas);

/* Scratch bytes ps_normalize needs for L matrices of rows x cols. */
PS_API int64_t ps_normalize_workspace_bytes(int64_t L, int64_t rows, int64_t cols);

/* xh[l] = fp16( fp32(x[l]) / (||fp32(x[l])||_F + eps) ), per matrix.
 * x: (L, rows, cols) of x_dtype with element strides (sL, sR, sC).
 * xh: FP16 (L, rows_p, cols_p) contiguous with rows_p >= rows, cols_p >= cols;
 * the padding is written with zeros. Replaces polar_switch/__init__.py:34-35. */
PS_API int ps_normalize(const void* x, int x_dtype, int64_t L, int64_t rows, int64_t cols, int64_t sL,
                 int64_t sR, int64_t sC, float eps, void* xh, int64_t rows_p, int64_t cols_p,
                 void* workspace, int64_t workspace_bytes, void* stream);

/* Allocation-free variant of ps_normalize (no counterpart in the reference).
 *
 * For callers that cannot allocate device memory at the point of the call:
 * code running under another framework's memory pool that owns all device
 * memory, real-time loops that must not enter the CUDA allocator, or foreign
 * runtimes that hold device pointers but no allocator. Instead of a caller
 * workspace, the partial sums live in a static scratch array inside the
 * library, PS_NORMALIZE_NOALLOC_MAX_PARTIALS doubles (256 KiB), which every
 * GPU that loads the library keeps until the process exits.
 *
 * Same arguments as ps_normalize without the workspace. While the L matrices'
 * partial sums (ps_normalize's chunking) fit the scratch, the result is the
 * same bits as ps_normalize; beyond that each matrix is summed over fewer,
 * longer chunks, which can move an output by one FP16 rounding step. L must
 * be at most PS_NORMALIZE_NOALLOC_MAX_PARTIALS (PS_ERR_UNSUPPORTED otherwise).
 * Calls no allocating routine. The first call on a device looks up the
 * scratch's device address (cudaGetSymbolAddress), so make that first call
 * before any stream capture. All calls on a device share the scratch: calls
 * whose kernels overlap on the GPU (different streams, no ordering) race and
 * give wrong results; calls ordered on one stream are safe. Every call writes
 * all the partial sums it reads, so leftovers of earlier calls never matter. */
#define PS_NORMALIZE_NOALLOC_MAX_PARTIALS 32768
PS_API int ps_normalize_noalloc(const void* x, int x_dtype, int64_t L, int64_t rows, int64_t cols,
                                int64_t sL, int64_t sR, int64_t sC, float eps, void* xh,
                                int64_t rows_p, int64_t cols_p, void* stream);

/* out = x @ x^T (rows <= cols) or x^T @ x (rows > cols), FP32 accumulate,
 * one FP16 rounding; out is (L, n, n) contiguous, n = min(rows, cols), n % 8 == 0.
 * Replaces gram() of polar_switch/gemm_symmetric_fused.py:291-293. */
PS_API int ps_gram(const void* x, void* out, int64_t L, int64_t rows, int64_t cols, int64_t x_ld,
            void* stream);

/* out = fp16(alpha * a @ a + beta * c + diag * I) for symmetric a; out may be
 * c but not a; c may be NULL (no addend). (L, n, n) contiguous, n % 8 == 0.
 * Replaces square() of polar_switch/gemm_symmetric_fused.py:296-301. */
PS_API int ps_square(const void* a, const void* c, void* out, int64_t L, int64_t n, float alpha,
              float beta, float diag, void* stream);

/* out = fp16(alpha * p @ q + beta * c + diag * I) for symmetric, commuting p
 * and q (so the product is symmetric): tiles on and above the block diagonal
 * are computed as p @ q and mirrored below it; out may be c but neither p nor
 * q; c may be NULL.
 * Replaces sym_baddbmm of polar_switch/gram_newton_schulz.py:64-72. */
PS_API int ps_sym_product(const void* p, const void* q, const void* c, void* out, int64_t L, int64_t n,
                   float alpha, float beta, float diag, void* stream);

/* y = b @ x + residual * x (rows <= cols) or x @ b + residual * x (rows > cols),
 * FP32 accumulate, one FP16 rounding, stored as y_dtype (PS_F16, PS_F32 or
 * PS_BF16; wider types are the FP16 value widened). b: (L, n, n) contiguous
 * (any square matrix: the product is exactly b @ x or x @ b); x: (L, rows, cols)
 * FP16 with pitch x_ld; y: pitch y_ld elements
 * (y_ld * sizeof(y_dtype) % 16 == 0). y must not overlap x or b.
 * Replaces apply() of polar_switch/gemm_symmetric_fused.py:304-309. */
PS_API int ps_apply(const void* b, const void* x, void* y, int64_t L, int64_t rows, int64_t cols,
             int64_t x_ld, float residual, int y_dtype, int64_t y_ld, void* stream);

/* out = fp16(in + fp16(a) * I), (L, n, n) contiguous; out may equal in.
 * Replaces `Z + a * I` of polar_switch/gram_newton_schulz.py:107. */
PS_API int ps_add_diag(const void* in, void* out, int64_t L, int64_t n, float a, void* stream);

/* Scratch bytes ps_circuit needs for L matrices of rows x cols and `buffers`
 * square buffers. */
PS_API int64_t ps_circuit_workspace_bytes(int64_t L, int64_t rows, int64_t cols, int buffers);

/* Whole Polar Switch circuit (polar_switch/__init__.py:25-45 plus the output
 * cast of :168): normalise x, then for each outer iteration t
 *   B[0] = gram(X); for each step: B[w] = a B[i]@B[i] + b B[r] + c I;
 *   X = B[w_last] @ X + residual_t X   (X @ B[w_last] + ... for rows > cols)
 * and write y (L, rows, cols) contiguous in y_dtype (any PS_* code).
 * x: (L, rows, cols) of x_dtype with element strides (sL, sR, sC).
 * Table: n_outer outer iterations; outer t has n_steps[t] consecutive entries
 * of `steps`; `buffers` square buffers. Validated like
 * polar_switch/__init__.py:107-122 (PS_ERR_INVALID on a bad table). */
PS_API int ps_circuit(const void* x, int x_dtype, int64_t L, int64_t rows, int64_t cols, int64_t sL,
               int64_t sR, int64_t sC, void* y, int y_dtype, int n_outer,
               const float* residuals, const int32_t* n_steps, const ps_step* steps, int buffers,
               float eps, void* workspace, int64_t workspace_bytes, void* stream);

/* One problem of a grouped circuit: x (L, rows, cols) of x_dtype with element
 * strides (sL, sR, sC); y (L, rows, cols) contiguous of y_dtype. */
typedef struct ps_problem {
  const void* x;
  int32_t x_dtype;
  int64_t L, rows, cols, sL, sR, sC;
  void* y;
  int32_t y_dtype;
} ps_problem;

/* Scratch bytes ps_circuit_grouped needs for these problems. */
PS_API int64_t ps_circuit_grouped_workspace_bytes(const ps_problem* probs, int n_probs, int buffers);

/* The circuit of ps_circuit applied to several problems of different shapes
 * (the buckets of a Muon step, reference training/muon.py:59-86), in one call:
 * the inner iterations of all problems that share n = min(rows, cols) run as
 * one batched launch per inner iteration. Same table and errors as ps_circuit. */
PS_API int ps_circuit_grouped(const ps_problem* probs, int n_probs, int n_outer,
                              const float* residuals, const int32_t* n_steps, const ps_step* steps,
                              int buffers, float eps, void* workspace, int64_t workspace_bytes,
                              void* stream);

/* A Muon update applied in place of storing a problem's result: for every
 * matrix l of the problem, p[l] <- fl(fl(p[l] * decay) + alpha * fl(u[l])),
 * u the circuit's result in the problem's y_dtype, rounded to p_dtype where
 * torch rounds it (training/muon.py:84-86: p.mul_(1 - lr * wd);
 * p.add_(u.to(p.dtype), alpha=-lr * scale)). p: (L, rows, cols) contiguous
 * bank of p_dtype (PS_F32, PS_BF16 or PS_F16). p == NULL: store y as usual. */
typedef struct ps_update {
  void* p;
  int p_dtype;
  float decay, alpha;
} ps_update;

/* ps_circuit_grouped, with the Muon update of problem i folded into its last
 * apply when updates[i].p is set: the update never exists in memory, the
 * parameter bank is read and written once in that kernel's epilogue (y of
 * that problem is not written and may be NULL). Needs the CTA-pair kernel
 * (ps_set_cta_pairs(1), the default), an unpadded problem (rows and cols
 * multiples of 8, contiguous) and a 16-byte aligned bank whose rows are a
 * multiple of 16 bytes; PS_ERR_UNSUPPORTED otherwise. No single counterpart in
 * the reference: it replaces orthogonalize-then-update (training/muon.py:
 * 77-86, train_nanogpt.py's sharded bank update) for banks of stacked
 * matrices. */
PS_API int ps_circuit_grouped_update(const ps_problem* probs, const ps_update* updates, int n_probs,
                                     int n_outer, const float* residuals, const int32_t* n_steps,
                                     const ps_step* steps, int buffers, float eps, void* workspace,
                                     int64_t workspace_bytes, void* stream);

/* ps_circuit_grouped in one whole-circuit launch whose final results are
 * also stored straight into other GPUs' memory: the all-gather after a
 * sharded orthogonalization (train_nanogpt.py:4025-4037, each rank's updates
 * all-gathered after its local orthogonalization) fused into the last
 * apply's epilogue, tile by tile, while later matrices still compute.
 *
 * Every y lies inside one buffer that starts at local_base on this GPU and
 * whose copy on peer k (the same layout) starts at peer_bases[k], a device
 * address this GPU can store to (a peer's symmetric-memory buffer); each
 * final tile is stored to y and, with 16-byte vector stores, to
 * peer_bases[k] + (y - local_base) for k < n_peers (at most 7). The stores
 * are complete when the kernel has finished;
 * ordering them against the peers' use of their buffers (a barrier before and
 * after the call) is the caller's. n_phases (1..8) groups each problem's
 * matrices: phase_ends[i * n_phases + k] is the number of problem i's matrices
 * in phases 0..k (non-decreasing, the last equal to its L; NULL when
 * n_phases == 1); the tiles of a phase are scheduled before those of the
 * next, so its results reach the peers while later phases compute. The bits
 * stored are ps_circuit_grouped's. Needs the whole-circuit kernel (at most 8
 * problems, ps_set_circuit_kernel(1)) and rows and cols multiples of 8 with
 * 16-byte aligned y and 16-byte rows; PS_ERR_UNSUPPORTED otherwise, before
 * anything is launched. */
PS_API int ps_circuit_grouped_push(const ps_problem* probs, int n_probs, int n_outer,
                                   const float* residuals, const int32_t* n_steps,
                                   const ps_step* steps, int buffers, float eps, void* workspace,
                                   int64_t workspace_bytes, const void* local_base,
                                   const void* const* peer_bases, int n_peers, int n_phases,
                                   const int32_t* phase_ends, void* stream);

/* ps_circuit_grouped in one whole-circuit launch, scheduled in phases like
 * ps_circuit_grouped_push, that raises a flag in device memory as soon as
 * every final result of a phase is stored: signals[k] becomes 1 (k <
 * n_phases) -- for another stream to start moving that phase's results
 * (copy engines: ps_stream_wait_flag, then peer copies) while the launch
 * computes the next phases, the all-gather of train_nanogpt.py:4025-4037
 * overlapping the circuit without splitting it into launches.
 * signals: PS_SIGNAL_WORDS(n_phases) 32-bit words of device memory, 16-byte
 * aligned, ZEROED BY THE CALLER before the launch in an order the waiting
 * stream observes (the words after the flags are the kernel's counters). The
 * last CTA to finish raises every flag, so a wait on them ends even if the
 * launch gave up early (ps_get_status then reports why). The bits stored are
 * ps_circuit_grouped's; same requirements as ps_circuit_grouped_push. */
#define PS_SIGNAL_WORDS(n_phases) (2 * (n_phases) + 1)
PS_API int ps_circuit_grouped_signal(const ps_problem* probs, int n_probs, int n_outer,
                                     const float* residuals, const int32_t* n_steps,
                                     const ps_step* steps, int buffers, float eps, void* workspace,
                                     int64_t workspace_bytes, int n_phases,
                                     const int32_t* phase_ends, unsigned* signals, void* stream);

/* Enqueues on `stream` a wait until the 32-bit word at device address `flag`
 * is >= value (cuStreamWaitValue32, GEQ); work enqueued after it starts once
 * the word is written. No counterpart in the reference. */
PS_API int ps_stream_wait_flag(void* stream, const unsigned* flag, unsigned value);

/* Scratch bytes ps_gns needs for L matrices of rows x cols. */
PS_API int64_t ps_gns_workspace_bytes(int64_t L, int64_t rows, int64_t cols);

/* Gram Newton-Schulz on rectangular matrices (replaces the rectangular branch
 * of polar_switch/gram_newton_schulz.py:75-122): normalise, R = X X^T (X^T X
 * when rows > cols), then for iteration i with coeffs[3i..3i+2] = (a, b, c):
 * Z = c R R + b R; Q = Z + a I at i = 0 and at restarts, else Q = Q Z + a Q;
 * before the next iteration (unless it restarts) R = Z (R Z + a R) + a (R Z
 * + a R); iteration i in `resets` (i > 0) first sets X <- Q X and R from it.
 * y = Q X (X Q when tall). Every product is one tcgen05 launch with FP32
 * accumulation and one FP16 rounding. Square matrices are rejected
 * (PS_ERR_INVALID): the reference sends them to Polar Express. */
PS_API int ps_gns(const void* x, int x_dtype, int64_t L, int64_t rows, int64_t cols, int64_t sL,
                  int64_t sR, int64_t sC, void* y, int y_dtype, int n_iter, const float* coeffs,
                  int n_resets, const int32_t* resets, float eps, void* workspace,
                  int64_t workspace_bytes, void* stream);

/* Pieces of the normalisation and of the Gram for a matrix split by columns
 * (or, tall, by rows) across ranks, the split Muon step for banks with fewer
 * matrices than ranks (no single counterpart in the reference; together they
 * replace polar_switch/__init__.py:34-35 and the Gram of :41 when the partial
 * results are summed across ranks between the calls):
 *   ps_sumsq: sums[l] = sum of squares of x[l] (FP64, the same chunks and
 *     order as ps_normalize); workspace of ps_normalize_workspace_bytes;
 *   ps_scale_cast: xh[l] = fp16(x[l] / (sqrt(sums[l]) + eps)), padding zeroed;
 *     sums == NULL gives a plain FP16 rounding (denominator 1);
 *   ps_gram_f32: out[l] = X X^T (X^T X when rows > cols) in FP32, not rounded,
 *     all n x n elements (general tiles). */
PS_API int ps_sumsq(const void* x, int x_dtype, int64_t L, int64_t rows, int64_t cols, int64_t sL,
                    int64_t sR, int64_t sC, double* sums, void* workspace, int64_t workspace_bytes,
                    void* stream);
PS_API int ps_scale_cast(const void* x, int x_dtype, int64_t L, int64_t rows, int64_t cols,
                         int64_t sL, int64_t sR, int64_t sC, const double* sums, float eps, void* xh,
                         int64_t rows_p, int64_t cols_p, void* stream);
PS_API int ps_gram_f32(const void* x, float* out, int64_t L, int64_t rows, int64_t cols,
                       int64_t x_ld, void* stream);

/* Muon's step before the circuit for one bucket of `count` same-shape matrices
 * of `elems` elements (replaces the momentum / Nesterov / stack / cast loop
 * of training/muon.py:63-74): for every matrix i, with grads[i] and moms[i]
 * device pointers of `dtype` (FP32, BF16 or FP16):
 *   m <- fl(fl(m * mu) + g);  d = fl(g + mu * m) (nesterov) or m;
 *   out[i] = d cast to out_dtype, out being (count, elems) contiguous.
 * The momentum buffers are updated in place; m and d are rounded to `dtype`
 * where torch rounds them. `grads` and `moms` are host arrays of pointers. */
PS_API int ps_muon_direction(const void* const* grads, void* const* moms, int count, int64_t elems,
                             int dtype, float mu, int nesterov, void* out, int out_dtype,
                             void* stream);

/* Muon's step after the circuit for one bucket (replaces training/muon.py:84-86):
 * for every matrix i (params[i] a device pointer of `dtype`, updates a
 * (count, elems) contiguous array of `upd_dtype`):
 *   p <- fl(fl(p * decay) + alpha * fl(u[i]))   decay = 1 - lr * wd,
 *                                               alpha = -lr * scale factor,
 * rounding to `dtype` where torch rounds. `params` is a host array. */
PS_API int ps_muon_update(void* const* params, int count, int64_t elems, int dtype,
                          const void* updates, int upd_dtype, float decay, float alpha,
                          void* stream);

/* Telemetry of orthogonalized updates (replaces the three passes of
 * training/diagnostics.py:161-165, NormLog.record): for each of L matrices of
 * `elems` contiguous elements of x_dtype (FP16, BF16 or FP32), in one pass,
 *   nan_count[l] = number of NaN entries, inf_count[l] = number of infinite
 *   entries, max_abs[l] = max |x| over the entries that are not NaN
 *   (infinity if any entry is infinite, 0 if every entry is NaN).
 * The three outputs are device arrays of L elements, overwritten. */
PS_API int ps_update_stats(const void* x, int x_dtype, int64_t L, int64_t elems, int64_t* nan_count,
                           int64_t* inf_count, float* max_abs, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* POLAR_SWITCH_B200_H */
