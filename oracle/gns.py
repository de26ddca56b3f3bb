"""CPU oracle of Gram Newton-Schulz (GNS) -- TEST INFRASTRUCTURE ONLY.

Restates the reference recurrence (polar_switch/gram_newton_schulz.py:80-118):
for X with n <= m, R = X X^T; per iteration i with quintic (a, b, c)

    Z = c*R@R + b*R                      (symmetric product, one rounding)
    Q = Z + a*I                          first iteration / after a restart
    Q = Q@Z + a*Q                        otherwise
    RZ = R@Z + a*R;  R = Z@RZ + a*RZ     unless the next iteration restarts

and at a restart X <- Q@X and R is recomputed; finally X <- Q@X (tall X uses
X^T X and X@Q). Every product is accumulated in `acc` precision and rounded
once to FP16. With mirror=True the symmetric products keep one triangle, as
the reference's QuACK gemm_symmetric does; mirror=False matches its PyTorch
backend (full products).
"""

import torch

from . import circuit as oc


def _mm(A, B, acc):
    return (A.to(acc) @ B.to(acc)).half()


def _sym(P, Q, C, alpha, beta, acc, mirror):
    D = alpha * (P.to(acc) @ Q.to(acc)) + beta * C.to(acc)
    return (oc._mirror_upper(D) if mirror else D).half()


def gns_run(X, coefficients, reset_iterations=(2,), epsilon=1e-7, acc=torch.float32, mirror=True):
    """Evaluate the GNS recurrence on rectangular X (..., rows, cols)."""
    shape, dtype = X.shape, X.dtype
    W = X.reshape(-1, *shape[-2:])
    Xh = oc.normalize(W, epsilon)
    tall = Xh.shape[-2] > Xh.shape[-1]
    resets = set(reset_iterations)

    def gram(Y):
        zero = torch.zeros(())
        return _sym(Y.mT, Y, zero, 1.0, 0.0, acc, mirror) if tall else _sym(Y, Y.mT, zero, 1.0, 0.0, acc, mirror)

    R = gram(Xh)
    n = R.shape[-1]
    eye = torch.eye(n, dtype=torch.float16)
    Q = None
    for i, (a, b, c) in enumerate(coefficients):
        if i in resets and i != 0:
            Xh = _mm(Xh, Q, acc) if tall else _mm(Q, Xh, acc)
            R = gram(Xh)
            Q = None
        Z = _sym(R, R, R, c, b, acc, mirror)
        if i == 0 or i in resets:
            Q = Z + a * eye
        else:
            Q = _sym(Q, Z, Q, 1.0, a, acc, mirror)
        if i < len(coefficients) - 1 and i + 1 not in resets:
            RZ = _sym(R, Z, R, 1.0, a, acc, mirror)
            R = _sym(Z, RZ, RZ, 1.0, a, acc, mirror)
    Xh = _mm(Xh, Q, acc) if tall else _mm(Q, Xh, acc)
    return Xh.to(dtype).reshape(shape)
