"""Telemetry of orthogonalized updates on the GPU: spectral-norm estimates and
non-finite counts, logged in the reference's format.

The reference (training/diagnostics.py) estimates each matrix's spectral norm
with Lanczos iterations on AᵀA that never form the Gram matrix: every
iteration reads an FP32 copy of A twice (q·Aᵀ, then ·A). Here the n × n Gram
(n = min(rows, cols)) is formed once on the tensor cores (ps_gram_f32, FP32
accumulation of the update scaled to max |x| = 1 and held in FP16), and the
iterations run on it: a 1024 × 3072 update costs 4 MB of reads per
iteration instead of 25 MB. The non-finite counts and max |x| come from one
pass over the update (ps_update_stats) instead of three.

Lanczos here keeps the whole Krylov basis and reorthogonalizes every new
vector against it (twice, classical Gram-Schmidt), so no eigenvalue is found
twice; the tridiagonal projection is solved in FP64. The estimate and its
checks follow the reference's contract (training/diagnostics.py:38-121):
the estimate is ||A v|| for the top Ritz vector v of the best probe, the
Ritz residual is ||AᵀA v - θ v|| / θ with θ = ||A v||², convergence is tested
every 16 iterations (residual <= rtol and relative change <= rtol / 4), and a
test counts as assessed from iteration 32 on.

Accuracy: for FP16 and BF16 updates the scaled FP16 copy is exact (to
FP16's subnormal range), and the estimate carries the Gram's FP32
accumulation error (~1e-4 relative); FP32 updates are rounded to FP16 first
(2^-11 per element), which moves the estimate by well under the default
rtol of 1e-3.
"""

import gzip
import json
import math
import time
from pathlib import Path

import torch

from . import cuda_ops

CHECK_EVERY = 16
START_SEED = 1729


def _tridiagonal(alpha, beta):
    """(…, k, k) symmetric tridiagonal matrices from diagonals alpha (…, k)
    and off-diagonals beta (…, k - 1)."""
    T = torch.diag_embed(alpha)
    if beta.shape[-1]:
        off = torch.diag_embed(beta, offset=1)
        T = T + off + off.mT
    return T


@torch.no_grad()
def lanczos_gram(G, rtol=1e-3, probes=4, max_iter=96, n_valid=None, seed=START_SEED):
    """Largest-eigenvalue estimates of a batch of symmetric positive
    semidefinite matrices G (B, n, n), returned as square roots: the spectral
    norms of the A with AᵀA = G.

    `probes` unit start vectors (fixed random, the same for every matrix, zero
    beyond `n_valid` coordinates) each run Lanczos with full
    reorthogonalization; the best probe's Ritz value is the estimate. Returns
    (estimates (B,), info) with info as the reference's spectral_norm.
    Runs on the device of G.
    """
    if G.ndim != 3 or G.shape[-1] != G.shape[-2]:
        raise ValueError("Expected a batch of square matrices")
    if rtol <= 0 or probes < 1 or max_iter < CHECK_EVERY:
        raise ValueError("Use positive tolerance/probes and at least 16 iterations")
    G = G.float()
    B, n, _ = G.shape
    n_valid = n if n_valid is None else int(n_valid)
    P = min(probes, n_valid)
    gen = torch.Generator(device=G.device).manual_seed(seed)
    start = torch.zeros(P, n, device=G.device, dtype=torch.float32)
    start[:, :n_valid] = torch.randn(P, n_valid, device=G.device, dtype=torch.float32, generator=gen)
    q = (start / start.norm(dim=-1, keepdim=True)).expand(B, P, n).contiguous()
    basis = torch.zeros(B, P, max_iter, n, device=G.device, dtype=torch.float32)
    alpha = torch.zeros(B, P, max_iter, device=G.device, dtype=torch.float32)
    beta = torch.zeros(B, P, max_iter, device=G.device, dtype=torch.float32)
    zero = G.abs().amax(dim=(-2, -1)) == 0
    last = torch.zeros(B, device=G.device)
    estimate = residual = change = torch.zeros(B, device=G.device)
    converged = zero.clone()
    iteration = 0
    for k in range(max_iter):
        iteration = k + 1
        basis[:, :, k] = q
        z = torch.matmul(q, G)  # (G q)ᵀ, G symmetric
        a = (z * q).sum(-1)
        alpha[:, :, k] = a
        V = basis[:, :, :k + 1]
        for _ in range(2):  # full reorthogonalization, twice
            z = z - torch.einsum("bpkn,bpk->bpn", V, torch.einsum("bpkn,bpn->bpk", V, z))
        b = z.norm(dim=-1)
        # an invariant subspace (b ~ 0 against the spectrum seen so far) ends the probe
        alive = b > 64 * torch.finfo(torch.float32).eps * alpha[:, :, :k + 1].abs().amax(-1).clamp_min(1e-30)
        beta[:, :, k] = torch.where(alive, b, torch.zeros_like(b))
        q = torch.where(alive.unsqueeze(-1), z / b.clamp_min(1e-30).unsqueeze(-1), torch.zeros_like(z))
        if iteration % CHECK_EVERY and iteration != max_iter:
            continue
        T = _tridiagonal(alpha[:, :, :iteration].double(), beta[:, :, :iteration - 1].double())
        _, vectors = torch.linalg.eigh(T)
        y = vectors[..., -1].float()  # (B, P, k) top Ritz vector coordinates
        ritz = torch.einsum("bpkn,bpk->bpn", V, y)
        ritz = ritz / ritz.norm(dim=-1, keepdim=True).clamp_min(1e-30)
        Gr = torch.matmul(ritz, G)
        theta = (Gr * ritz).sum(-1).clamp_min(0)  # ||A v||^2
        cand = theta.sqrt()
        estimate, best = cand.max(dim=-1)
        res_all = (Gr - theta.unsqueeze(-1) * ritz).norm(dim=-1) / theta.clamp_min(1e-30)
        residual = res_all.gather(-1, best[:, None]).squeeze(-1)
        change = (estimate - last).abs() / estimate.clamp_min(1e-30)
        converged = ((residual <= rtol) & (change <= rtol * 0.25)) | zero
        last = estimate
        if bool(converged.all()):
            break
    assessed = torch.full_like(converged, iteration >= 2 * CHECK_EVERY) | zero
    reported_change = torch.where(assessed, change, torch.full_like(change, float("nan")))
    estimate = torch.where(zero, torch.zeros_like(estimate), estimate)
    return estimate, dict(converged=converged, convergence_assessed=assessed, iterations=iteration,
                          ritz_residual=residual, relative_change=reported_change,
                          projection_fp64_retries=0)


@torch.no_grad()
def spectral_norm(x, rtol=1e-3, probes=4, max_iter=96):
    """Spectral-norm estimates of a batch of finite matrices x (B, rows, cols)
    on the GPU, with the reference's return value: (estimates, info dict with
    converged, convergence_assessed, iterations, ritz_residual,
    relative_change, projection_fp64_retries)."""
    if x.ndim != 3 or not x.is_floating_point() or min(x.shape) < 1:
        raise ValueError("Expected a nonempty batch of real floating matrices")
    if not x.is_cuda:
        raise NotImplementedError("spectral_norm: polar_switch_b200 runs on CUDA tensors only")
    B, rows, cols = x.shape
    _, _, scale = cuda_ops.update_stats(x if x.dtype != torch.float64 else x.float())
    unit = torch.where(scale > 0, scale, torch.ones_like(scale))
    rp, cp = -(-rows // 8) * 8, -(-cols // 8) * 8
    xh = torch.zeros(B, rp, cp, device=x.device, dtype=torch.float16)
    xh[:, :rows, :cols] = (x.float() / unit[:, None, None]).half()
    G = cuda_ops.gram_f32(xh)  # over the columns when rp > cp, else over the rows
    valid = cols if rp > cp else rows
    estimate, info = lanczos_gram(G, rtol=rtol, probes=probes, max_iter=max_iter, n_valid=valid)
    return estimate * scale, info


class NormLog:
    """Per-matrix spectral-norm estimates and non-finite counts of
    orthogonalized updates, written to compressed JSONL.

    The file, its metadata record and its per-batch records are those of the
    reference's NormLog (training/diagnostics.py:123-199), so tools that read
    its logs read these. `stats` and `estimator` default to the GPU
    implementations (cuda_ops.update_stats, spectral_norm).
    """

    def __init__(self, path, rank, method, stats=None, estimator=None):
        path = Path(path)
        path.mkdir(parents=True, exist_ok=True)
        self.step = 0
        self.method = method
        self.stats = stats or cuda_ops.update_stats
        self.estimator = estimator or spectral_norm
        self.path = path / f"rank-{rank:04d}-{time.time_ns()}.jsonl.gz"
        self.stream = gzip.open(self.path, "xt", compresslevel=1)
        self.stream.write(json.dumps(dict(
            event="metadata", format="polar-output-norm-v2", method=method, rank=rank,
            estimator="Lanczos", probes=1, max_iter=64, rtol=0.001,
            estimate_only=True, stage="post_orthogonalization_before_optimizer_scaling",
            step_index="zero-based, excludes warmup")) + "\n")

    @torch.no_grad()
    def record(self, label, output, matrix_start=0, execution=None, matrix_names=None):
        """Record one batch of orthogonalized matrices (…, rows, cols). Matrices
        with non-finite entries are counted, not estimated; an estimator
        failure is recorded, not raised."""
        mats = output.detach().reshape(-1, *output.shape[-2:])
        nan_count, inf_count, max_abs = self.stats(mats)
        ok = (nan_count == 0) & (inf_count == 0)
        blank = torch.full((len(mats),), float("nan"), device=mats.device)
        per_matrix = {"spectral_norm": blank.clone(), "ritz_residual": blank.clone(),
                      "relative_change": blank.clone()}
        flags = {"converged": torch.zeros(len(mats), dtype=torch.bool, device=mats.device),
                 "convergence_assessed": torch.zeros(len(mats), dtype=torch.bool, device=mats.device)}
        iterations, retries, error = 0, 0, None
        if bool(ok.any()):
            try:
                estimate, info = self.estimator(mats[ok], probes=1, max_iter=64, rtol=0.001)
            except torch.linalg.LinAlgError as exc:  # a diagnostic failure keeps the update
                error = str(exc)
            else:
                per_matrix["spectral_norm"][ok] = estimate.float()
                for key in ("ritz_residual", "relative_change"):
                    per_matrix[key][ok] = info[key].float()
                for key in flags:
                    flags[key][ok] = info[key]
                iterations, retries = info["iterations"], info["projection_fp64_retries"]

        def json_floats(t):
            return [v if math.isfinite(v) else None for v in t.float().cpu().tolist()]

        rec = {
            "event": "orthogonalization", "step": self.step, "label": label,
            "matrix_start": matrix_start, "matrix_names": matrix_names, "shape": list(mats.shape),
            "dtype": str(output.dtype), "requested": self.method, "execution": execution,
            "spectral_norm": json_floats(per_matrix["spectral_norm"]), "max_abs": json_floats(max_abs),
            "nan_count": nan_count.cpu().tolist(), "inf_count": inf_count.cpu().tolist(),
            "converged": flags["converged"].cpu().tolist(),
            "convergence_assessed": flags["convergence_assessed"].cpu().tolist(),
            "ritz_residual": json_floats(per_matrix["ritz_residual"]),
            "relative_change": json_floats(per_matrix["relative_change"]),
            "iterations": iterations, "projection_fp64_retries": retries, "estimator_error": error,
        }
        self.stream.write(json.dumps(rec, allow_nan=False, separators=(",", ":")) + "\n")
        if self.step % 32 == 31:
            self.stream.flush()

    def close(self):
        """Close the log file."""
        self.stream.close()
