"""CPU oracle of the Polar Switch circuit -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
module, always as the checker; the product (polar_switch) never imports it.

It restates the reference evaluator (polar_switch/__init__.py:25-45) with the
rounding rule the circuits were designed for (reference README.md "Rounding";
polar_switch/README.md:7-17): every gram / inner iteration / apply is one
contraction accumulated in `acc` precision (FP32 primary, FP64 secondary), the
alpha, beta*C and c*I terms are added in that precision, and the result is
rounded once to FP16. Symmetric products keep one triangle and mirror it, as
the reference kernels do (polar_switch/triton_kernels.py:50-57,
polar_switch/gemm_symmetric_fused.py:45-49).

Pinning: tests/test_oracle.py checks this module against golden vectors made
by the reference's own Triton kernels (run on CPU under TRITON_INTERPRET=1 by
tests/golden/make_golden.py) and against the published singular-value
intervals (reference README.md:64-73).
"""

import torch


def frobenius_norm_f32(X):
    """||X||_F of FP32 matrices, rounded once to FP32 from an FP64 sum.

    The reference takes torch's FP32 norm of a CUDA tensor (a tree reduction,
    within an ulp or two of the exact value). Torch's FP32 norm on the CPU
    drifts far more on large matrices (about 6e-5 relative at 3M elements),
    so the oracle rounds the exact norm instead.
    """
    return X.double().pow(2).sum(dim=(-2, -1), keepdim=True).sqrt().float()


def normalize(X, epsilon):
    """fp16(fp32(X) / (||fp32(X)||_F + eps)) per matrix (reference __init__.py:34-35)."""
    X = X.float()
    return (X / (frobenius_norm_f32(X) + epsilon)).half().contiguous()


TILE = 128


def _mirror_upper(D, tile=TILE):
    """Keep the tiles on and above the block diagonal and mirror them below.

    The kernels own square tiles of `tile` rows: a diagonal tile is computed
    in full, an off-diagonal tile above the diagonal is computed and also
    stored transposed below it (the reference Triton kernel does the same with
    128-row tiles, polar_switch/triton_kernels.py:44-57). For an exactly
    symmetric product this equals the plain product up to FP32 rounding.
    """
    n = D.shape[-1]
    blk = torch.arange(n) // tile
    keep = blk.unsqueeze(1) <= blk.unsqueeze(0)  # tile row <= tile column
    return torch.where(keep, D, D.mT)


def gram(X, tall, acc=torch.float32):
    """fp16(X @ X.T) or fp16(X.T @ X) for tall X (reference gemm_symmetric_fused.py:291-293)."""
    Xa = X.to(acc)
    G = Xa.mT @ Xa if tall else Xa @ Xa.mT
    return _mirror_upper(G).half()


def square(A, C, alpha, beta, diag, acc=torch.float32):
    """fp16(alpha*A@A + beta*C + diag*I) (reference gemm_symmetric_fused.py:296-301)."""
    Aa = A.to(acc)
    D = alpha * (Aa @ Aa.mT)
    if C is not None:
        D = D + beta * C.to(acc)
    if diag != 0:
        n = A.shape[-1]
        D = D + diag * torch.eye(n, dtype=acc)
    return _mirror_upper(D).half()


def sym_product(P, Q, C=None, alpha=1.0, beta=1.0, diag=0.0, acc=torch.float32):
    """fp16(alpha*P@Q + beta*C + diag*I) for symmetric commuting P, Q (one triangle)."""
    D = alpha * (P.to(acc) @ Q.to(acc))
    if C is not None:
        D = D + beta * C.to(acc)
    if diag != 0:
        D = D + diag * torch.eye(P.shape[-1], dtype=acc)
    return _mirror_upper(D).half()


def apply(X, B, tall, residual, acc=torch.float32):
    """fp16(B@X + residual*X) or fp16(X@B + residual*X) for tall X (reference :304-309)."""
    Xa, Ba = X.to(acc), B.to(acc)
    D = Xa @ Ba if tall else Ba @ Xa
    if residual != 0:
        D = D + residual * Xa
    return D.half()


def add_diag(Z, a):
    """torch's `Z + a * I` in FP16: fp16(Z_ii + fp16(a)) on the diagonal."""
    eye = torch.eye(Z.shape[-1], dtype=torch.float16)
    return Z + a * eye


def run_circuit(X, table, epsilon=1e-7, acc=torch.float32, out_dtype=None):
    """Evaluate a coefficient table on X (..., rows, cols); returns out_dtype (default X.dtype)."""
    shape, dtype = X.shape, X.dtype
    W = X.reshape(-1, *shape[-2:])
    Xh = normalize(W, epsilon)
    tall = Xh.shape[-2] > Xh.shape[-1]
    nbuf = 1 + max(max(w, i, r) for _, steps in table for w, i, r, *_ in steps)
    work = [None] * nbuf
    for residual, steps in table:
        work[0] = gram(Xh, tall, acc)
        for dst, src, add, alpha, beta, diag in steps:
            work[dst] = square(work[src], work[add], alpha, beta, diag, acc)
        Xh = apply(Xh, work[steps[-1][0]], tall, residual, acc)
    return Xh.to(out_dtype or dtype).reshape(shape)


def relative_frobenius(A, B):
    """||A - B||_F / ||B||_F per batch, in FP64 (max over the batch)."""
    A = A.double().reshape(-1, *A.shape[-2:])
    B = B.double().reshape(-1, *B.shape[-2:])
    num = torch.linalg.matrix_norm(A - B)
    den = torch.linalg.matrix_norm(B).clamp_min(1e-300)
    return float((num / den).max())


def singular_interval(Y):
    """(min sigma, max sigma) over every matrix of Y, computed in FP64."""
    s = torch.linalg.svdvals(Y.double().reshape(-1, *Y.shape[-2:]))
    return float(s.min()), float(s.max())
