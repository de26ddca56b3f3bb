"""Gram Newton-Schulz (GNS) on B200 kernels.

Same method and dispatch as the reference (polar_switch/gram_newton_schulz.py):
for X with n <= m the recurrence forms R = X X^T once and applies each quintic
multiplier h_t(z) = a_t + b_t z + c_t z^2 to R instead of X; Q accumulates the
multipliers since the last restart; at a restart X <- Q X and R is formed
again; finally X <- Q X. Tall matrices use X^T X and X Q. The package's GNS
uses the Polar Express preset with a restart after iteration 2 and its last
quintic centred so the final interval is centred at one. Square inputs use
POLAR_EXPRESS.

Every product here is one tcgen05 kernel with FP32 accumulation and one FP16
rounding: symmetric products (R R, Q Z, R Z, Z RZ, which commute) compute one
triangle of tiles and mirror it (ps_sym_product), X products use ps_apply,
and Q = Z + a I uses ps_add_diag.
"""

import math

import torch

from . import cuda_ops

# Polar Express preset of the upstream GNS implementation, divided by the
# safety factor 1.05 (reference polar_switch/gram_newton_schulz.py:33-44).
_UNMODIFIED_POLAR_EXPRESS_COEFFICIENTS = [
    (8.28721201814563, -23.595886519098837, 17.300387312530933),
    (4.107059111542203, -2.9478499167379106, 0.5448431082926601),
    (3.9486908534822946, -2.908902115962949, 0.5518191394370137),
    (3.3184196573706015, -2.488488024314874, 0.51004894012372),
    (2.300652019954817, -1.6689039845747493, 0.4188073119525673),
]
SAFETY_FACTOR = 1.05
POLAR_EXPRESS_COEFFICIENTS = [
    (a / SAFETY_FACTOR, b / SAFETY_FACTOR ** 3, c / SAFETY_FACTOR ** 5)
    for (a, b, c) in _UNMODIFIED_POLAR_EXPRESS_COEFFICIENTS
]
# The package's GNS: the last quintic scaled by 2 / (L + U) = 1.0795859163621828
# (reference polar_switch/gram_newton_schulz.py:45-50).
GNS_COEFFICIENTS = POLAR_EXPRESS_COEFFICIENTS[:-1] + [
    (2.365477637327074, -1.5563980023821433, 0.3542623265416755),
]
RESET_ITERATIONS = (2,)


def gns_flops(rows, cols, batch=1):
    """Algorithmic FLOPs of the GNS method, (6 alpha + 14) n^3 (reference README)."""
    n, m = min(rows, cols), max(rows, cols)
    return float((6 * (m / n) + 14) * n ** 3) * batch


def gram_newton_schulz(X, coefficients=GNS_COEFFICIENTS, reset_iterations=RESET_ITERATIONS,
                       epsilon=1e-7):
    """Run the GNS recurrence on CUDA X (..., rows, cols) as one library call
    (ps_gns: workspace, padding of dimensions that are not multiples of 8 and
    the output cast all inside it); returns X's dtype and shape."""
    import ctypes

    from . import _native as nat
    if not isinstance(X, torch.Tensor) or not X.is_cuda:
        raise NotImplementedError("gram_newton_schulz: polar_switch_b200 runs on CUDA tensors only")
    shape, dtype = X.shape, X.dtype
    if dtype not in nat.DTYPE_CODES:
        raise TypeError(f"Unsupported dtype {dtype}")
    W = X.reshape(-1, *shape[-2:])
    L, rows, cols = W.shape
    Y = torch.empty(W.shape, device=X.device, dtype=dtype)
    flat = [float(v) for abc in coefficients for v in abc]
    coeffs = (ctypes.c_float * len(flat))(*flat)
    resets = (ctypes.c_int32 * max(len(reset_iterations), 1))(*reset_iterations)
    lib = nat.load()
    with torch.cuda.device(X.device):
        ws_bytes = lib.ps_gns_workspace_bytes(L, rows, cols)
        if ws_bytes < 0:
            nat.check("ps_gns_workspace_bytes", ws_bytes)
        ws = torch.empty(ws_bytes, device=X.device, dtype=torch.uint8)
        sL, sR, sC = W.stride()
        nat.check("ps_gns", lib.ps_gns(
            nat.ptr(W), nat.DTYPE_CODES[dtype], L, rows, cols, sL, sR, sC, nat.ptr(Y),
            nat.DTYPE_CODES[dtype], len(coefficients), coeffs, len(reset_iterations), resets,
            float(epsilon), nat.ptr(ws), ws_bytes, nat.stream_ptr(X.device)))
    return Y.reshape(shape)


def gram_newton_schulz_ops(X, coefficients=GNS_COEFFICIENTS, reset_iterations=RESET_ITERATIONS,
                           epsilon=1e-7):
    """The same recurrence op by op through the public kernels (full, mirrored
    n x n buffers); kept as the step-by-step form of `gram_newton_schulz`,
    which must give the same bits."""
    shape, dtype = X.shape, X.dtype
    Xh = cuda_ops.normalize(X.reshape(-1, *shape[-2:]), epsilon)
    tall = Xh.shape[-2] > Xh.shape[-1]
    n = min(Xh.shape[-2:])
    resets = set(reset_iterations)

    def gram(Y):
        R = torch.empty((Y.shape[0], n, n), device=Y.device, dtype=torch.float16)
        return cuda_ops.gram(Y, tall, R)

    def times_q(Y, Q, out_dtype=torch.float16):
        return cuda_ops.apply(Y, Q, tall, 0.0, out_dtype=out_dtype)

    R = gram(Xh)
    Q = None
    last = len(coefficients) - 1
    for i, (a, b, c) in enumerate(coefficients):
        if i in resets and i != 0:
            Xh = times_q(Xh, Q)
            R = gram(Xh)
            Q = None
        Z = cuda_ops.sym_product(R, R, R, alpha=c, beta=b)
        if i == 0 or i in resets:
            Q = cuda_ops.add_diag(Z, a)
        else:
            Q = cuda_ops.sym_product(Q, Z, Q, alpha=1.0, beta=a)
        if i < last and i + 1 not in resets:
            RZ = cuda_ops.sym_product(R, Z, R, alpha=1.0, beta=a)
            R = cuda_ops.sym_product(Z, RZ, RZ, alpha=1.0, beta=a)
    out_dtype = dtype if dtype in (torch.float16, torch.float32, torch.bfloat16) else torch.float16
    Y = times_q(Xh, Q, out_dtype)
    return Y.to(dtype).reshape(shape)


def make_orthogonalizer(pe_factory, compile=True, epsilon=1e-7):
    """Create the GNS orthogonalizer (reference polar_switch/gram_newton_schulz.py:276-357).

    Rectangular inputs run the centred Gram recurrence; square inputs use
    POLAR_EXPRESS from ``pe_factory`` (make_polynomial_orthogonalizer).
    ``last_execution`` records ``dispatch``: ``rectangular_gram`` or
    ``square_polar_express``. There is no fallback path, so
    ``fallback_polar_express`` never occurs and ``fallback_events`` stays empty.
    """
    from . import BACKEND, _check_input

    if not math.isfinite(epsilon) or epsilon <= 0:
        raise ValueError("Use a positive finite epsilon")
    pe = pe_factory("POLAR_EXPRESS", compile=compile, epsilon=epsilon)

    flat_coeffs = [float(v) for abc in GNS_COEFFICIENTS for v in abc]

    def polar(X, out=None):
        """Approximate the polar factor of each matrix in X."""
        _check_input(X)
        compiling = torch.compiler.is_compiling()
        if X.shape[-2] == X.shape[-1]:
            result = pe(X, out=out)
            if not compiling:
                polar.last_execution = dict(pe.last_execution, requested="GNS",
                                            dispatch="square_polar_express")
            return result
        if compiling:
            # Traced by torch.compile: one polar_switch::gns operator, no
            # attribute updates (provenance is recorded by eager calls).
            result = torch.ops.polar_switch.gns(X, flat_coeffs, list(RESET_ITERATIONS), float(epsilon))
            if out is not None:
                out.copy_(result)
                result = out
            return result
        result = gram_newton_schulz(X, epsilon=epsilon)
        if out is not None:
            out.copy_(result)
            result = out
        polar.last_execution = dict(requested="GNS", effective="GNS", backend=BACKEND,
                                    dispatch="rectangular_gram")
        return result

    polar.fallback_events = pe.fallback_events
    polar.last_execution = None
    polar.method = "GNS"
    polar.epsilon = epsilon
    return polar
