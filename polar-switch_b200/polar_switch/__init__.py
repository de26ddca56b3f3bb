"""Polar Switch matrix orthogonalization on NVIDIA B200 (sm_100a).

Drop-in for the reference package's public API (reference:
polar_switch/__init__.py:20-186):

    from polar_switch import make_polynomial_orthogonalizer, METHODS
    orthogonalize = make_polynomial_orthogonalizer("PS2_55")
    update = orthogonalize(G)          # G: CUDA tensor (..., rows, cols)

A method is a sequence of outer iterations. Each forms the Gram matrix of X,
runs its inner iterations ``B[w] = a*B[i]@B[i] + b*B[r] + c*I`` on two or
three square FP16 buffers, and multiplies the last buffer into X. Every
contraction is one hand-written tcgen05 kernel with FP32 accumulation and one
FP16 rounding (libpolarswitch_b200.so, C ABI in include/polar_switch_b200.h).

Differences from the reference, by design: there is one backend (the B200
kernels), so nothing falls back; CPU tensors and non-B200 devices raise
instead of silently running Polar Express. ``fallback_events`` therefore stays
empty and ``last_execution`` records backend ``"b200"``.
"""

import ctypes
import math

import torch

from . import _native as nat
from . import coefficients

# Method names accepted by make_polynomial_orthogonalizer (same set and order
# as the reference, polar_switch/__init__.py:21-22).
METHODS = ("JORDAN", "POLAR_EXPRESS", "GNS", "PS2_55", "PS2_64", "PS2_54", "PS2_512",
           "PS2_4111", "PS2_11111", "PS3_55", "PS3_64", "PS3_54")

BACKEND = "b200"

__all__ = ["METHODS", "make_polynomial_orthogonalizer", "coefficients", "circuit_flops"]


def _run(X, table, ops, epsilon, buffers):
    """Evaluate a coefficient table op by op with an ``ops`` module.

    Same structure as the reference's evaluator (polar_switch/__init__.py:25-45):
    normalise in FP32 and store FP16, then per outer iteration gram -> inner
    iterations -> apply. ``ops`` provides normalize, gram, square and apply
    (``polar_switch.cuda_ops``). The fused path used by the orthogonalizer is
    ``_Circuit``, which issues the same kernels from one C call.
    """
    X = ops.normalize(X, epsilon)
    tall = X.shape[-2] > X.shape[-1]
    n = min(X.shape[-2:])
    work = [torch.empty((*X.shape[:-2], n, n), device=X.device, dtype=X.dtype)
            for _ in range(buffers)]
    for residual, steps in table:
        ops.gram(X, tall, work[0])
        for dst, src, add, alpha, beta, diag in steps:
            ops.square(work[src], work[add], work[dst], alpha, beta, diag)
        X = ops.apply(X, work[steps[-1][0]], tall, residual)
    return X


def validate_table(table, epsilon):
    """Check a coefficient table like the reference (polar_switch/__init__.py:107-122).

    Returns the number of square buffers the circuit needs.
    """
    if not math.isfinite(epsilon) or epsilon <= 0 or not table:
        raise ValueError("Use a nonempty circuit and positive finite epsilon")
    buffers = 1
    for residual, steps in table:
        initialized = {0}
        if not steps or not math.isfinite(residual):
            raise ValueError("Each outer iteration needs a finite residual and at least one inner iteration")
        for dst, src, add, alpha, beta, diag in steps:
            if (any(not isinstance(i, int) or i < 0 for i in (dst, src, add))
                    or dst == src or src not in initialized or add not in initialized
                    or not all(math.isfinite(v) for v in (alpha, beta, diag))):
                raise ValueError("Invalid inner iteration: buffer indices must be nonnegative integers, the "
                                 "destination must differ from the squared buffer, operands must be B[0] "
                                 "or buffers written earlier, and coefficients must be finite")
            initialized.add(dst)
            buffers = max(buffers, dst + 1, src + 1, add + 1)
    return buffers


def circuit_flops(table, rows, cols, batch=1):
    """Algorithmic FLOPs of one evaluation, counted as the reference does.

    Symmetric products count n^3 (half of 2n^3), the Gram n^2 m and the apply
    2 n^2 m per outer iteration: sum_t (3 alpha + k_t) n^3 with alpha = m / n
    (reference README, FLOP column: PS-55 = (6 alpha + 10) n^3).
    """
    n, m = min(rows, cols), max(rows, cols)
    per = sum(3 * n * n * m + len(steps) * n ** 3 for _, steps in table)
    return float(per) * batch


class _Circuit:
    """A validated table packed for ps_circuit (C structs built once)."""

    def __init__(self, table, buffers):
        self.buffers = buffers
        self.n_outer = len(table)
        flat = [st for _, steps in table for st in steps]
        self.residuals = (ctypes.c_float * self.n_outer)(*[float(r) for r, _ in table])
        self.n_steps = (ctypes.c_int32 * self.n_outer)(*[len(steps) for _, steps in table])
        self.steps = (nat.PsStep * len(flat))(
            *[nat.PsStep(int(w), int(i), int(r), float(a), float(b), float(c)) for w, i, r, a, b, c in flat])

    def __call__(self, X, epsilon, out=None):
        """Run the whole circuit on X (..., rows, cols); returns X's dtype and shape."""
        if X.dtype not in nat.DTYPE_CODES:
            raise TypeError(f"Unsupported dtype {X.dtype}; use float16/bfloat16/float32/float64")
        work = X.reshape(-1, *X.shape[-2:])
        L, rows, cols = work.shape
        if out is None:
            out = torch.empty(X.shape, device=X.device, dtype=X.dtype)
        elif out.shape != X.shape or out.dtype != X.dtype or not out.is_contiguous() or out.device != X.device:
            raise ValueError("out must be a contiguous tensor with the shape, dtype and device of X")
        lib = nat.load()
        with torch.cuda.device(X.device):
            ws_bytes = lib.ps_circuit_workspace_bytes(L, rows, cols, self.buffers)
            if ws_bytes < 0:
                nat.check("ps_circuit_workspace_bytes", nat.PS_ERR_INVALID)
            ws = torch.empty(ws_bytes, device=X.device, dtype=torch.uint8)
            sL, sR, sC = work.stride()
            nat.check("ps_circuit", lib.ps_circuit(
                nat.ptr(work), nat.DTYPE_CODES[X.dtype], L, rows, cols, sL, sR, sC,
                nat.ptr(out), nat.DTYPE_CODES[X.dtype], self.n_outer, self.residuals, self.n_steps,
                self.steps, self.buffers, float(epsilon), nat.ptr(ws), ws_bytes,
                nat.stream_ptr(X.device)))
        return out


    def grouped(self, banks, epsilon, outs=None, updates=None, push=None, signal=None):
        """Run the circuit on several tensors of different shapes in one C call.

        Tensors that share n = min(rows, cols) have their inner iterations
        batched into one launch each. Returns one output per input (its dtype
        and shape unless ``outs`` supplies tensors, which may be FP16 to
        receive the circuit's FP16 result without widening).

        ``updates``: optional list with, per input, None or a tuple
        ``(param_bank, decay, alpha)``: the result u of that input is not
        returned but applied as ``p <- p * decay + alpha * u`` (Muon's update,
        rounded as torch's ``p.mul_(decay); p.add_(u.to(p.dtype), alpha)``) to
        the contiguous bank of the input's shape, inside the last apply
        (ps_circuit_grouped_update). Its entry in the returned list is None.

        ``push``: optional dict ``{"local": int, "peers": [int, ...],
        "phase_ends": [[int, ...], ...]}``: every output lies in a buffer
        starting at device address ``local`` whose copies on other GPUs start
        at ``peers``; the final results are also stored there, tile by tile,
        inside the circuit's one launch (ps_circuit_grouped_push), the
        matrices of each input scheduled in the phases ``phase_ends[i]``
        (cumulative counts ending at the input's matrix count). Raises
        NativeError (PS_ERR_UNSUPPORTED, before anything ran) when the inputs
        do not fit that launch.

        ``signal``: optional dict ``{"flags": int32 device tensor of
        2 * phases + 1 words, zeroed by the caller, "phase_ends": [...]}``:
        one launch scheduled in those phases that sets ``flags[k]`` to 1 once
        phase k's results are stored (ps_circuit_grouped_signal), for another
        stream to wait on (``_native.stream_wait_flag``).
        """
        if not banks:
            return []
        lib = nat.load()
        device = banks[0].device
        works, results = [], []
        probs = (nat.PsProblem * len(banks))()
        upd = None
        if updates is not None:
            upd = (nat.PsUpdate * len(banks))()
        for i, X in enumerate(banks):
            if X.device != device:
                raise ValueError("all tensors of a grouped call must be on one device")
            if X.dtype not in nat.DTYPE_CODES:
                raise TypeError(f"Unsupported dtype {X.dtype}")
            W = X.reshape(-1, *X.shape[-2:])
            target = updates[i] if updates is not None else None
            if target is not None:
                P, decay, alpha = target
                if (P.shape != X.shape or not P.is_contiguous() or P.device != device
                        or P.dtype not in (torch.float32, torch.bfloat16, torch.float16)):
                    raise ValueError("an update target must be a contiguous FP32/BF16/FP16 bank of "
                                     "its input's shape on the same device")
                upd[i] = nat.PsUpdate(P.data_ptr(), nat.DTYPE_CODES[P.dtype], float(decay), float(alpha))
                Y = None
            else:
                Y = outs[i] if outs is not None else torch.empty(X.shape, device=device, dtype=X.dtype)
                if Y.shape != X.shape or not Y.is_contiguous() or Y.dtype not in nat.DTYPE_CODES:
                    raise ValueError("each output must be contiguous with its input's shape")
            works.append(W)
            results.append(Y)
            L, rows, cols = W.shape
            sL, sR, sC = W.stride()
            probs[i] = nat.PsProblem(W.data_ptr(), nat.DTYPE_CODES[X.dtype], L, rows, cols, sL, sR, sC,
                                     Y.data_ptr() if Y is not None else None,
                                     nat.DTYPE_CODES[Y.dtype if Y is not None else X.dtype])
        with torch.cuda.device(device):
            ws_bytes = lib.ps_circuit_grouped_workspace_bytes(probs, len(banks), self.buffers)
            if ws_bytes < 0:
                nat.check("ps_circuit_grouped_workspace_bytes", nat.PS_ERR_INVALID)
            ws = torch.empty(ws_bytes, device=device, dtype=torch.uint8)
            if signal is not None:
                if upd is not None or push is not None:
                    raise ValueError("signal cannot be combined with push or updates")
                ends = signal.get("phase_ends")
                n_phases = len(ends[0]) if ends else 1
                if ends and any(len(e) != n_phases for e in ends):
                    raise ValueError("every input needs the same number of phases")
                flags = signal["flags"]
                if flags.device != device or flags.numel() < 2 * n_phases + 1:
                    raise ValueError("flags must hold 2 * phases + 1 words on the inputs' device")
                flat = [int(v) for e in ends for v in e] if ends else []
                nat.check("ps_circuit_grouped_signal", lib.ps_circuit_grouped_signal(
                    probs, len(banks), self.n_outer, self.residuals, self.n_steps, self.steps,
                    self.buffers, float(epsilon), nat.ptr(ws), ws_bytes, n_phases,
                    (ctypes.c_int32 * max(1, len(flat)))(*flat) if flat else None,
                    nat.ptr(flags), nat.stream_ptr(device)))
            elif push is not None:
                if upd is not None:
                    raise ValueError("push and updates cannot be combined")
                peers = [int(p) for p in push.get("peers", ())]
                ends = push.get("phase_ends")
                n_phases = len(ends[0]) if ends else 1
                if ends and any(len(e) != n_phases for e in ends):
                    raise ValueError("every input needs the same number of phases")
                flat = [int(v) for e in ends for v in e] if ends else []
                nat.check("ps_circuit_grouped_push", lib.ps_circuit_grouped_push(
                    probs, len(banks), self.n_outer, self.residuals, self.n_steps, self.steps,
                    self.buffers, float(epsilon), nat.ptr(ws), ws_bytes, push.get("local"),
                    (ctypes.c_void_p * max(1, len(peers)))(*peers), len(peers), n_phases,
                    (ctypes.c_int32 * max(1, len(flat)))(*flat) if flat else None,
                    nat.stream_ptr(device)))
            elif upd is None:
                nat.check("ps_circuit_grouped", lib.ps_circuit_grouped(
                    probs, len(banks), self.n_outer, self.residuals, self.n_steps, self.steps,
                    self.buffers, float(epsilon), nat.ptr(ws), ws_bytes, nat.stream_ptr(device)))
            else:
                nat.check("ps_circuit_grouped_update", lib.ps_circuit_grouped_update(
                    probs, upd, len(banks), self.n_outer, self.residuals, self.n_steps, self.steps,
                    self.buffers, float(epsilon), nat.ptr(ws), ws_bytes, nat.stream_ptr(device)))
        return results


def _check_input(X):
    if not isinstance(X, torch.Tensor) or X.ndim < 2 or X.numel() == 0 or not X.is_floating_point():
        raise ValueError("Expected nonempty real matrices")
    if not X.is_cuda:
        raise NotImplementedError(
            "polar_switch_b200 runs on CUDA (B200) tensors only; there is no CPU fallback")


def make_polynomial_orthogonalizer(method, compile=True, epsilon=1e-7):
    """Create an orthogonalizer for a named method or a coefficient table.

    Args:
        method: A name in METHODS, such as "PS2_55" (case-insensitive), or a
            coefficient table in the format of coefficients.py.
        compile: Accepted for API compatibility. The kernels are compiled
            ahead of time, so there is nothing to trace; the value is ignored.
        epsilon: Added to the Frobenius norm before normalization.

    Returns:
        A callable that accepts a real floating point CUDA tensor with shape
        (..., rows, columns) and returns its approximate polar factor with the
        same shape and dtype. The input is not modified. Attributes
        ``fallback_events`` (always empty: there is no fallback) and
        ``last_execution`` (requested/effective method and backend).

    "GNS" returns the Gram Newton-Schulz orthogonalizer of
    polar_switch.gram_newton_schulz (square inputs use POLAR_EXPRESS).
    """
    if isinstance(method, str) and method.upper() == "GNS":
        from .gram_newton_schulz import make_orthogonalizer
        return make_orthogonalizer(make_polynomial_orthogonalizer, compile, epsilon)
    table = method
    if isinstance(method, str):
        if method.upper() not in METHODS:
            raise ValueError(f"Unknown method: {method}")
        table = getattr(coefficients, method.upper())
    name = next((n for n in METHODS if n != "GNS" and table == getattr(coefficients, n)), "CUSTOM")
    buffers = validate_table(table, epsilon)
    circuit = _Circuit(table, buffers)
    events = []

    from . import torch_ops
    op_args = torch_ops.table_to_lists(table)

    def polar(X, out=None):
        """Approximate the polar factor of each matrix in X."""
        _check_input(X)
        if torch.compiler.is_compiling():
            # Traced by torch.compile: one polar_switch::circuit operator, no
            # attribute updates (provenance is recorded by eager calls).
            result = torch.ops.polar_switch.circuit(X, *op_args, buffers, float(epsilon))
            if out is not None:
                out.copy_(result)
                result = out
            return result
        result = circuit(X, epsilon, out=out)
        polar.last_execution = dict(requested=name, effective=name, backend=BACKEND)
        return result

    def grouped(tensors, outs=None, updates=None, push=None, signal=None):
        """Orthogonalize a list of tensors of different shapes in one grouped call
        (``updates``: fold Muon's update of a parameter bank into the last apply;
        ``push``: also store the results into other GPUs' buffers from inside
        the circuit's launch; see _Circuit.grouped)."""
        for X in tensors:
            _check_input(X)
        result = circuit.grouped(list(tensors), epsilon, outs=outs, updates=updates, push=push,
                                 signal=signal)
        polar.last_execution = dict(requested=name, effective=name, backend=BACKEND)
        return result

    polar.grouped = grouped
    polar.fallback_events = events
    polar.last_execution = None
    polar.table = table
    polar.method = name
    polar.buffers = buffers
    polar.epsilon = epsilon
    return polar


# Registers the polar_switch:: operators used under torch.compile.
from . import torch_ops  # noqa: E402,F401
