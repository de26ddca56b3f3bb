"""Helpers shared by the test modules (seeded inputs, FP16 comparisons)."""

import math

import torch


def seeded(shape, seed, dtype=torch.float32, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g, dtype=torch.float64) * scale).to(dtype)


def haar(n, k, gen):
    """First k columns of an n x n Haar-random orthogonal matrix (QR with sign fix)."""
    Z = torch.randn(n, k, generator=gen, dtype=torch.float64)
    Q, R = torch.linalg.qr(Z)
    return Q * torch.sign(torch.diagonal(R)).unsqueeze(0)


def log_uniform_matrix(rows, cols, seed, lo=1e-3, hi=1.0, batch=None):
    """X = U diag(s) V^T with Haar U, V and s log-uniform on [lo, hi]."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(batch or 1):
        n = min(rows, cols)
        U = haar(rows, n, g)
        V = haar(cols, n, g)
        s = torch.exp(torch.empty(n, dtype=torch.float64).uniform_(math.log(lo), math.log(hi), generator=g))
        out.append((U * s) @ V.T)
    X = torch.stack(out)
    return X if batch else X[0]


def fp16_ulp(x):
    """Spacing of FP16 numbers at |x| (subnormal spacing near zero)."""
    a = x.abs().float().clamp_min(2.0 ** -14)
    e = torch.floor(torch.log2(a))
    return torch.pow(2.0, e - 10)


def assert_fp16_close(got, ref, max_ulps=1, max_mismatch=0.02, what="", terms=None, k=None):
    """Element-wise FP16 agreement up to `max_ulps` rounding flips.

    Two FP32-accumulated products rounded once to FP16 may land on adjacent
    FP16 values when their FP32 sums differ in the last bits; anything larger
    is a kernel error.

    With `terms` (the magnitude |alpha * acc| + |beta * C| + |diag| of what
    the epilogue adds, per element) and `k` (the contraction length), an
    element may also differ by k * 2^-26 of its terms: the tensor cores'
    FP32 accumulation is not IEEE round-to-nearest (partial sums are aligned
    and truncated), so over a long K its error, relative to the terms, grows
    to ~(k / 16) * 2^-24. That only matters where the epilogue cancels and the
    result is far smaller than its terms (FP16 subnormals near zero); the
    oracle itself (IEEE FP32 on the CPU) agrees with an FP64 evaluation to
    1 ulp everywhere.
    """
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    assert torch.isfinite(got).all(), f"{what}: non-finite output"
    diff = (got - ref).abs()
    tol = max_ulps * fp16_ulp(ref) + 1e-7 * ref.abs().max()
    if terms is not None:
        tol = tol + float(k) * 2.0 ** -26 * terms.detach().float().cpu()
    bad = diff > tol
    worst = float((diff / fp16_ulp(ref)).max())
    if bad.any():
        idx = bad.nonzero()[:4].tolist()
        detail = "; ".join(f"{tuple(i)}: ref {float(ref[tuple(i)]):.6g} got {float(got[tuple(i)]):.6g}"
                           + (f" terms {float(terms[tuple(i)]):.3g}" if terms is not None else "")
                           for i in idx)
        raise AssertionError(f"{what}: {int(bad.sum())} elements beyond {max_ulps} ulp "
                             f"(worst {worst:.2f} ulp): {detail}")
    frac = float((diff > 0).float().mean())
    assert frac <= max_mismatch, f"{what}: {frac:.4f} of elements differ (limit {max_mismatch})"
    return frac
