"""torch.library custom operators around the B200 library, so the
orthogonalizers and the op-level backend compose with torch.compile
(fullgraph=True) without graph breaks.

The reference registers its fused QuACK kernel the same way
(polar_switch/gemm_symmetric_fused.py:211-244): an out-variant operator that
mutates `out`, with a fake implementation describing it to the compiler, and
an ``accumulate`` flag instead of passing the same tensor as both the addend
and the output (a mutated argument may not alias another input).

Operators (all CUDA-only; their fake versions only describe shapes):

    polar_switch::circuit(X, residuals, n_steps, steps, buffers, epsilon) -> Y
        a whole coefficient table on X (..., rows, cols), Y with X's dtype;
        the table travels as flat lists (`steps`: 6 numbers per inner step)
    polar_switch::gns(X, coeffs, resets, epsilon) -> Y
        the rectangular Gram Newton-Schulz recurrence
    polar_switch::normalize(X, epsilon) -> Xh (FP16)
    polar_switch::gram_out(X, tall, out) -> ()
    polar_switch::square_out(A, out, C, alpha, beta, diag, accumulate) -> ()
    polar_switch::apply(X, B, tall, residual) -> X' (FP16)

`compiled_ops` is a backend module for ``_run`` whose gram/square/apply go
through these operators.
"""

import types
from typing import List, Optional

import torch
from torch import Tensor

from . import cuda_ops

_CIRCUITS = {}


def table_to_lists(table):
    """(residuals, n_steps, steps) of a coefficient table, the operator's encoding."""
    residuals = [float(r) for r, _ in table]
    n_steps = [len(steps) for _, steps in table]
    flat = [float(v) for _, steps in table for st in steps for v in st]
    return residuals, n_steps, flat


def _lists_to_table(residuals, n_steps, steps):
    table, k = [], 0
    for r, count in zip(residuals, n_steps):
        inner = []
        for _ in range(count):
            w, i, a, alpha, beta, diag = steps[6 * k:6 * k + 6]
            inner.append((int(w), int(i), int(a), alpha, beta, diag))
            k += 1
        table.append((r, tuple(inner)))
    return tuple(table)


def _circuit(residuals, n_steps, steps, buffers):
    key = (tuple(residuals), tuple(n_steps), tuple(steps), int(buffers))
    c = _CIRCUITS.get(key)
    if c is None:
        from . import _Circuit
        c = _CIRCUITS[key] = _Circuit(_lists_to_table(residuals, n_steps, steps), int(buffers))
    return c


@torch.library.custom_op("polar_switch::circuit", mutates_args=(), device_types="cuda")
def circuit(X: Tensor, residuals: List[float], n_steps: List[int], steps: List[float],
            buffers: int, epsilon: float) -> Tensor:
    """Run a coefficient table on X; returns a new tensor with X's dtype and shape."""
    return _circuit(residuals, n_steps, steps, buffers)(X, epsilon)


@circuit.register_fake
def _circuit_fake(X, residuals, n_steps, steps, buffers, epsilon):
    return torch.empty(X.shape, dtype=X.dtype, device=X.device)


@torch.library.custom_op("polar_switch::gns", mutates_args=(), device_types="cuda")
def gns(X: Tensor, coeffs: List[float], resets: List[int], epsilon: float) -> Tensor:
    """Rectangular Gram Newton-Schulz; `coeffs` holds (a, b, c) per iteration."""
    from .gram_newton_schulz import gram_newton_schulz
    triples = [tuple(coeffs[3 * i:3 * i + 3]) for i in range(len(coeffs) // 3)]
    return gram_newton_schulz(X, triples, tuple(resets), epsilon)


@gns.register_fake
def _gns_fake(X, coeffs, resets, epsilon):
    return torch.empty(X.shape, dtype=X.dtype, device=X.device)


@torch.library.custom_op("polar_switch::normalize", mutates_args=(), device_types="cuda")
def normalize(X: Tensor, epsilon: float) -> Tensor:
    return cuda_ops.normalize(X, epsilon)


@normalize.register_fake
def _normalize_fake(X, epsilon):
    return torch.empty(X.shape, dtype=torch.float16, device=X.device)


@torch.library.custom_op("polar_switch::gram_out", mutates_args=("out",), device_types="cuda")
def gram_out(X: Tensor, tall: bool, out: Tensor) -> None:
    cuda_ops.gram(X, tall, out)


@gram_out.register_fake
def _gram_out_fake(X, tall, out):
    return None


@torch.library.custom_op("polar_switch::square_out", mutates_args=("out",), device_types="cuda")
def square_out(A: Tensor, out: Tensor, C: Optional[Tensor], alpha: float, beta: float, diag: float,
               accumulate: bool) -> None:
    """out = alpha*A@A + beta*(out if accumulate else C) + diag*I."""
    cuda_ops.square(A, out if accumulate else C, out, alpha, beta, diag)


@square_out.register_fake
def _square_out_fake(A, out, C, alpha, beta, diag, accumulate):
    return None


@torch.library.custom_op("polar_switch::apply", mutates_args=(), device_types="cuda")
def apply(X: Tensor, B: Tensor, tall: bool, residual: float) -> Tensor:
    return cuda_ops.apply(X, B, tall, residual)


@apply.register_fake
def _apply_fake(X, B, tall, residual):
    return torch.empty(X.shape, dtype=torch.float16, device=X.device)


def _gram(X, tall, out):
    torch.ops.polar_switch.gram_out(X, bool(tall), out)
    return out


def _square(A, C, out, alpha, beta, diag):
    accumulate = C is out
    torch.ops.polar_switch.square_out(A, out, None if accumulate else C, float(alpha), float(beta),
                                      float(diag), accumulate)
    return out


def _apply(X, B, tall, residual):
    return torch.ops.polar_switch.apply(X, B, bool(tall), float(residual))


def _normalize(X, epsilon):
    return torch.ops.polar_switch.normalize(X, float(epsilon))


# The backend-module interface of ``_run`` (normalize / gram / square / apply),
# through the operators.
compiled_ops = types.SimpleNamespace(normalize=_normalize, gram=_gram, square=_square, apply=_apply)
