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


def assert_fp16_close(got, ref, max_ulps=1, max_mismatch=0.02, what=""):
    """Element-wise FP16 agreement up to `max_ulps` rounding flips.

    Two FP32-accumulated products rounded once to FP16 may land on adjacent
    FP16 values when their FP32 sums differ in the last bits; anything larger
    is a kernel error.
    """
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    assert torch.isfinite(got).all(), f"{what}: non-finite output"
    diff = (got - ref).abs()
    tol = max_ulps * fp16_ulp(ref) + 1e-7 * ref.abs().max()
    bad = diff > tol
    worst = float((diff / fp16_ulp(ref)).max())
    assert not bad.any(), f"{what}: {int(bad.sum())} elements beyond {max_ulps} ulp (worst {worst:.2f} ulp)"
    frac = float((diff > 0).float().mean())
    assert frac <= max_mismatch, f"{what}: {frac:.4f} of elements differ (limit {max_mismatch})"
    return frac
