"""The three circuit operations on B200 tensor cores, plus the helpers around them.

This module has the duck-typed interface of the reference's backend modules
(polar_switch/gemm_symmetric_fused.py:291-309 and polar_switch/triton_kernels.py:72-87),
so ``_run(X, table, cuda_ops, epsilon, buffers)`` evaluates a circuit op by op:

    gram(X, tall, out)                        out = X @ X.T  (X.T @ X if tall)
    square(A, C, out, alpha, beta, diag)      out = alpha*A@A + beta*C + diag*I
    apply(X, B, tall, residual) -> X'         X' = B@X + residual*X  (X@B + ... if tall)

Each call is one launch of a hand-written sm_100a kernel through the C ABI
(FP16 operands, FP32 accumulation in TMEM, one FP16 rounding). Tensors must be
CUDA FP16 and contiguous; nothing falls back to another implementation.
"""

import torch

from . import _native as nat


def _require(t, name, dtype=torch.float16):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise NotImplementedError(f"{name}: polar_switch_b200 runs on CUDA tensors only")
    if t.dtype != dtype:
        raise TypeError(f"{name}: expected {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name}: expected a contiguous tensor")


def _batched(t):
    return t.reshape(-1, *t.shape[-2:])


def gram(X, tall, out):
    """Write X @ X.T, or X.T @ X for tall X, into out (FP16, FP32 accumulate)."""
    _require(X, "gram X")
    _require(out, "gram out")
    rows, cols = X.shape[-2:]
    if bool(tall) != (rows > cols):
        raise ValueError("gram: tall must equal rows > cols")
    n = cols if tall else rows
    if tuple(out.shape[-2:]) != (n, n) or out.numel() // (n * n) != X.numel() // (rows * cols):
        raise ValueError("gram: out must have shape (..., n, n)")
    L = X.numel() // (rows * cols)
    with torch.cuda.device(X.device):
        nat.check("ps_gram", nat.load().ps_gram(nat.ptr(X), nat.ptr(out), L, rows, cols, cols,
                                                nat.stream_ptr(X.device)))
    return out


def square(A, C, out, alpha, beta, diag):
    """Write alpha*A @ A + beta*C + diag*I into out; out may be C but not A."""
    return sym_product(A, A, C, out, alpha, beta, diag, _name="ps_square")


def sym_product(P, Q, C=None, out=None, alpha=1.0, beta=1.0, diag=0.0, _name="ps_sym_product"):
    """Return alpha*P@Q + beta*C + diag*I for symmetric, commuting P and Q.

    Only one triangle of tiles is computed and mirrored, as for a symmetric
    product (reference: polar_switch/gram_newton_schulz.py:64-72 sym_baddbmm).
    """
    _require(P, f"{_name} P")
    _require(Q, f"{_name} Q")
    n = P.shape[-1]
    if P.shape != Q.shape or P.shape[-2] != n:
        raise ValueError(f"{_name}: operands must be (..., n, n) of the same shape")
    if out is None:
        out = torch.empty_like(P)
    _require(out, f"{_name} out")
    if C is not None:
        _require(C, f"{_name} C")
        if C.shape != P.shape:
            raise ValueError(f"{_name}: C must have the operand shape")
    if out.shape != P.shape:
        raise ValueError(f"{_name}: out must have the operand shape")
    if out.data_ptr() in (P.data_ptr(), Q.data_ptr()):
        raise ValueError(f"{_name}: out may be C but not a multiplied operand")
    L = P.numel() // (n * n)
    lib = nat.load()
    with torch.cuda.device(P.device):
        s = nat.stream_ptr(P.device)
        if _name == "ps_square":
            rc = lib.ps_square(nat.ptr(P), nat.ptr(C), nat.ptr(out), L, n, float(alpha),
                               float(beta), float(diag), s)
        else:
            rc = lib.ps_sym_product(nat.ptr(P), nat.ptr(Q), nat.ptr(C), nat.ptr(out), L, n,
                                    float(alpha), float(beta), float(diag), s)
        nat.check(_name, rc)
    return out


def apply(X, B, tall, residual, out=None, out_dtype=torch.float16):
    """Return B @ X + residual*X, or X @ B + residual*X for tall X.

    The result is rounded once to FP16; ``out_dtype`` FP32/BF16 widens that
    FP16 value (the reference's final ``.to(X.dtype)``).
    """
    _require(X, "apply X")
    _require(B, "apply B")
    rows, cols = X.shape[-2:]
    if bool(tall) != (rows > cols):
        raise ValueError("apply: tall must equal rows > cols")
    n = cols if tall else rows
    L = X.numel() // (rows * cols)
    if tuple(B.shape[-2:]) != (n, n) or B.numel() // (n * n) != L:
        raise ValueError("apply: B must have shape (..., n, n)")
    if out is None:
        out = torch.empty(X.shape, device=X.device, dtype=out_dtype)
    _require(out, "apply out", out.dtype)
    if out.dtype not in (torch.float16, torch.float32, torch.bfloat16) or out.shape != X.shape:
        raise ValueError("apply: out must be FP16/FP32/BF16 with the shape of X")
    with torch.cuda.device(X.device):
        nat.check("ps_apply", nat.load().ps_apply(
            nat.ptr(B), nat.ptr(X), nat.ptr(out), L, rows, cols, cols, float(residual),
            nat.DTYPE_CODES[out.dtype], cols, nat.stream_ptr(X.device)))
    return out


def add_diag(Z, a, out=None):
    """Return Z + a*I with torch's FP16 semantics, fp16(Z_ii + fp16(a))."""
    _require(Z, "add_diag Z")
    if out is None:
        out = torch.empty_like(Z)
    _require(out, "add_diag out")
    n = Z.shape[-1]
    L = Z.numel() // (n * n)
    with torch.cuda.device(Z.device):
        nat.check("ps_add_diag", nat.load().ps_add_diag(nat.ptr(Z), nat.ptr(out), L, n, float(a),
                                                        nat.stream_ptr(Z.device)))
    return out


def normalize(X, epsilon, out=None):
    """Return fp16(fp32(X) / (||fp32(X)||_F + epsilon)) per matrix (contiguous).

    Reference: polar_switch/__init__.py:34-35. X may be FP16/BF16/FP32/FP64
    with any strides.
    """
    if not isinstance(X, torch.Tensor) or not X.is_cuda:
        raise NotImplementedError("normalize: polar_switch_b200 runs on CUDA tensors only")
    if X.dtype not in nat.DTYPE_CODES:
        raise TypeError(f"normalize: unsupported dtype {X.dtype}")
    W = _batched(X)
    L, rows, cols = W.shape
    if out is None:
        out = torch.empty(W.shape, device=X.device, dtype=torch.float16)
    lib = nat.load()
    with torch.cuda.device(X.device):
        ws_bytes = lib.ps_normalize_workspace_bytes(L, rows, cols)
        if ws_bytes < 0:
            nat.check("ps_normalize_workspace_bytes", nat.PS_ERR_INVALID)
        ws = torch.empty(max(ws_bytes, 16), device=X.device, dtype=torch.uint8)
        sL, sR, sC = W.stride()
        nat.check("ps_normalize", lib.ps_normalize(
            nat.ptr(W), nat.DTYPE_CODES[X.dtype], L, rows, cols, sL, sR, sC, float(epsilon),
            nat.ptr(out), rows, cols, nat.ptr(ws), ws_bytes, nat.stream_ptr(X.device)))
    return out.reshape(X.shape)


# ---------------------------------------------------------------- split matrices
# The pieces of a circuit whose matrix is split by columns (rows when tall)
# across ranks: the sums of squares and the Gram are partial on each rank and
# are summed across the ranks between these calls.

def sumsq(X):
    """Per-matrix sum of squares of X (..., rows, cols), any strides, as FP64 (L,)."""
    if not isinstance(X, torch.Tensor) or not X.is_cuda:
        raise NotImplementedError("sumsq: polar_switch_b200 runs on CUDA tensors only")
    if X.dtype not in nat.DTYPE_CODES:
        raise TypeError(f"sumsq: unsupported dtype {X.dtype}")
    W = _batched(X)
    L, rows, cols = W.shape
    sums = torch.empty(L, device=X.device, dtype=torch.float64)
    lib = nat.load()
    with torch.cuda.device(X.device):
        ws_bytes = lib.ps_normalize_workspace_bytes(L, rows, cols)
        ws = torch.empty(max(ws_bytes, 16), device=X.device, dtype=torch.uint8)
        sL, sR, sC = W.stride()
        nat.check("ps_sumsq", lib.ps_sumsq(nat.ptr(W), nat.DTYPE_CODES[X.dtype], L, rows, cols, sL, sR, sC,
                                            nat.ptr(sums), nat.ptr(ws), ws_bytes, nat.stream_ptr(X.device)))
    return sums


def scale_cast(X, sums, epsilon, out=None):
    """fp16(X / (sqrt(sums) + epsilon)) per matrix; ``sums`` None: plain FP16 rounding."""
    if not isinstance(X, torch.Tensor) or not X.is_cuda:
        raise NotImplementedError("scale_cast: polar_switch_b200 runs on CUDA tensors only")
    if X.dtype not in nat.DTYPE_CODES:
        raise TypeError(f"scale_cast: unsupported dtype {X.dtype}")
    W = _batched(X)
    L, rows, cols = W.shape
    if sums is not None:
        _require(sums, "scale_cast sums", torch.float64)
        if sums.numel() != L:
            raise ValueError("scale_cast: one sum per matrix")
    if out is None:
        out = torch.empty(W.shape, device=X.device, dtype=torch.float16)
    _require(out, "scale_cast out")
    with torch.cuda.device(X.device):
        sL, sR, sC = W.stride()
        nat.check("ps_scale_cast", nat.load().ps_scale_cast(
            nat.ptr(W), nat.DTYPE_CODES[X.dtype], L, rows, cols, sL, sR, sC,
            nat.ptr(sums) if sums is not None else None, float(epsilon), nat.ptr(out), rows, cols,
            nat.stream_ptr(X.device)))
    return out.reshape(X.shape)


def gram_f32(X, out=None):
    """X @ X.T (X.T @ X when tall) of FP16 X in FP32, not rounded, all n x n elements."""
    _require(X, "gram_f32 X")
    rows, cols = X.shape[-2:]
    n = min(rows, cols)
    L = X.numel() // (rows * cols)
    if out is None:
        out = torch.empty((*X.shape[:-2], n, n), device=X.device, dtype=torch.float32)
    _require(out, "gram_f32 out", torch.float32)
    with torch.cuda.device(X.device):
        nat.check("ps_gram_f32", nat.load().ps_gram_f32(nat.ptr(X), nat.ptr(out), L, rows, cols, cols,
                                                        nat.stream_ptr(X.device)))
    return out


def update_stats(X):
    """Per matrix of X (..., rows, cols): (NaN count, infinite count, max |x|)
    as int64, int64 and float32 tensors of shape X.shape[:-2], from one pass
    over X (ps_update_stats). Like torch's abs().amax(), max |x| is NaN for a
    matrix with a NaN entry and infinite for one with an infinite entry."""
    if not isinstance(X, torch.Tensor) or not X.is_cuda:
        raise NotImplementedError("update_stats: polar_switch_b200 runs on CUDA tensors only")
    if X.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise TypeError(f"update_stats: expected FP16, BF16 or FP32, got {X.dtype}")
    if X.ndim < 2 or X.numel() == 0:
        raise ValueError("update_stats: expected nonempty matrices")
    W = _batched(X.contiguous())
    L = W.shape[0]
    nan = torch.empty(L, device=X.device, dtype=torch.int64)
    inf = torch.empty(L, device=X.device, dtype=torch.int64)
    amax = torch.empty(L, device=X.device, dtype=torch.float32)
    with torch.cuda.device(X.device):
        nat.check("ps_update_stats", nat.load().ps_update_stats(
            nat.ptr(W), nat.DTYPE_CODES[X.dtype], L, W.shape[1] * W.shape[2], nat.ptr(nan), nat.ptr(inf),
            nat.ptr(amax), nat.stream_ptr(X.device)))
    amax = torch.where(nan > 0, torch.full_like(amax, float("nan")), amax)
    shape = X.shape[:-2]
    return nan.reshape(shape), inf.reshape(shape), amax.reshape(shape)
