"""The single-read normalisation inside circuits (ps_set_fused_normalize(1);
off by default, the two passes measured faster): each contiguous, unpadded
input is read once, a chunk kept in
shared memory until its matrix's norm is known. It sums the same chunks in the
same order as the two-pass kernels, so whole circuits must give the same bits
with it on and off, for every input type, for matrices of one chunk, of a
partial last chunk, of many chunks, batches of many small matrices, and inputs
that do not qualify (padded, strided, more chunks than the resident grid) and
take the two passes either way.
"""

import pytest
import torch

from polar_switch import _native as nat
from polar_switch import make_polynomial_orthogonalizer

pytestmark = pytest.mark.gpu


def _both(fn):
    prev = nat.set_fused_normalize(1)
    try:
        on = fn()
        torch.cuda.synchronize()
        nat.set_fused_normalize(0)
        off = fn()
        torch.cuda.synchronize()
    finally:
        nat.set_fused_normalize(prev)
    return on, off


CASES = [
    (torch.float32, [(3, 1024, 3072), (2, 2048, 1024), (4, 1024, 1024)]),  # Qwen-like banks
    (torch.bfloat16, [(5, 768, 768), (2, 768, 3072)]),
    (torch.float16, [(300, 64, 64), (7, 256, 512)]),                          # one chunk per matrix
    (torch.float64, [(2, 1000, 24), (1, 384, 1024)]),                         # a partial last chunk
    (torch.float32, [(3, 130, 66), (1, 4096, 4096)]),                          # padded; > 1024 chunks
]


@pytest.mark.parametrize("dtype,shapes", CASES, ids=[f"{str(d)[6:]}-{len(s)}" for d, s in CASES])
def test_fused_normalisation_gives_the_two_pass_bits(cuda_device, dtype, shapes):
    g = torch.Generator().manual_seed(31)
    banks = [(torch.randn(*s, generator=g) * 3.0).to(dtype).to(cuda_device) for s in shapes]
    polar = make_polynomial_orthogonalizer("PS2_55")
    on, off = _both(lambda: polar.grouped(banks))
    for a, b, s in zip(on, off, shapes):
        assert torch.equal(a, b), f"{dtype} {s}: fused and two-pass normalisation differ"
    assert nat.get_status() == 0


def test_fused_normalisation_strided_input_takes_two_passes(cuda_device):
    X = torch.randn(2, 512, 768, device=cuda_device).mT  # (2, 768, 512), not contiguous
    polar = make_polynomial_orthogonalizer("PS3_55")
    on, off = _both(lambda: polar(X))
    assert torch.equal(on, off)
