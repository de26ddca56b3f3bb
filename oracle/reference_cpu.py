"""Port of the reference's CPU path -- TEST INFRASTRUCTURE / CPU BASELINE ONLY.

On a CPU tensor the reference orthogonalizer runs POLAR_EXPRESS, whatever
method was requested, with torch.bmm/baddbmm on FP16 tensors and no fused
rounding (reference polar_switch/__init__.py:48-63 `_TorchPE`, :125-126
`torch_pe`, :180-182 the final fallback). This module restates that path so
bench.py can time it on the GPU box's host cores (where the reference project
is not installed) and the tests can check it against the golden output of the
reference itself (tests/golden/cpu_path_ps2_55_128x256.npz).
"""

import torch

# POLAR_EXPRESS table as (residual, a, b) per outer iteration: one inner
# iteration B[1] = a*B[0]@B[0] + b*B[0]; X = B[1]@X + residual*X.
# Values: reference polar_switch/coefficients.py:26-32.
POLAR_EXPRESS_STEPS = (
    (8.156554524902461, 15.878769915207457, -22.483292925577953),
    (4.042929935166734, 0.500017845105131, -2.8089174659087113),
    (3.891667802292659, 0.506064817850339, -2.772484153217684),
    (3.2857536577556523, 0.4644902423300304, -2.3681294933425354),
    (2.3465413258596395, 0.42323551169305257, -1.709782838268708),
)


def torch_pe(X, epsilon=1e-7):
    """The reference CPU fallback on X (..., rows, cols); returns X's dtype and shape."""
    shape, dtype = X.shape, X.dtype
    W = X.reshape(-1, *shape[-2:]).float()
    W = (W / (W.norm(dim=(-2, -1), keepdim=True) + epsilon)).half().contiguous()
    tall = W.shape[-2] > W.shape[-1]
    n = min(W.shape[-2:])
    B0 = torch.empty((W.shape[0], n, n), dtype=W.dtype)
    B1 = torch.empty_like(B0)
    for residual, a, b in POLAR_EXPRESS_STEPS:
        torch.bmm(W.mT, W, out=B0) if tall else torch.bmm(W, W.mT, out=B0)
        torch.baddbmm(B0, B0, B0, alpha=a, beta=b, out=B1)
        W = torch.baddbmm(W, W, B1, beta=residual) if tall else torch.baddbmm(W, B1, W, beta=residual)
    return W.to(dtype).reshape(shape)
