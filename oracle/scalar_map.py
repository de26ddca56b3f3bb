"""Scalar map of a circuit on singular values -- TEST INFRASTRUCTURE ONLY.

A circuit acts on each singular value x of the normalised input separately:
per outer iteration, B[0] = x^2, every inner iteration is the scalar
B[w] = a*B[i]^2 + b*B[r] + c, and x <- B[w_last]*x + residual*x
(reference polar_switch/__init__.py:25-45 restricted to diagonal matrices).
The final interval over x in [1e-3, 1] is the published accuracy figure
(reference README.md:64-73, polar_switch/README.md:31-44), which makes these
intervals known answers for the tables.
"""

import numpy as np


def circuit_map(table, x):
    """Apply a coefficient table to an array of scalars (float64)."""
    x = np.asarray(x, dtype=np.float64)
    for residual, steps in table:
        B = {0: x * x}
        last = 0
        for w, i, r, a, b, c in steps:
            B[w] = a * B[i] * B[i] + b * B[r] + c
            last = w
        x = B[last] * x + residual * x
    return x


def circuit_map_stored(table, x, factor):
    """circuit_map with every stored value multiplied by factor(shape): the
    Gram, each inner iteration's buffer and each outer iteration's output.
    This is the rounding model under which the reference certified its
    circuits' upper endpoints (coefficient_search/stage*.json "verification":
    every stored value times a factor in [1/safety, safety])."""
    x = np.asarray(x, dtype=np.float64)
    for residual, steps in table:
        B = {0: x * x * factor(x.shape)}
        last = 0
        for w, i, r, a, b, c in steps:
            B[w] = (a * B[i] * B[i] + b * B[r] + c) * factor(x.shape)
            last = w
        x = (B[last] * x + residual * x) * factor(x.shape)
    return x


def quintic_map(coefficients, x):
    """Compose quintics x <- a x + b x^3 + c x^5 (Gram Newton-Schulz steps)."""
    x = np.asarray(x, dtype=np.float64)
    for a, b, c in coefficients:
        x2 = x * x
        x = a * x + b * x * x2 + c * x * x2 * x2
    return x


def final_interval(fn, lo=1e-3, hi=1.0, points=2_000_001):
    """(min, max) of fn over a dense log grid of [lo, hi] plus local refinement."""
    x = np.exp(np.linspace(np.log(lo), np.log(hi), points))
    y = fn(x)
    out = []
    for arg in (np.argmin(y), np.argmax(y)):
        a = x[max(arg - 1, 0)]
        b = x[min(arg + 1, len(x) - 1)]
        xx = np.linspace(a, b, 20001)
        yy = fn(xx)
        out.append(yy.min() if arg == np.argmin(y) else yy.max())
    return float(out[0]), float(out[1])
