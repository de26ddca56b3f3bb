"""Parity at the sizes the performance claims are made on.

Op level (every element within 1 FP16 ulp of the FP32-accumulating oracle, a
few percent of elements allowed to differ by that one rounding flip; where a
square's epilogue cancels, the result may also differ by n * 2^-26 of the
magnitude of its terms, the tensor cores' truncating FP32 accumulation over
K = n -- see tests/_util.assert_fp16_close):
  * symmetric products with more than 16 row blocks of 128 (n > 2048), on CTA
    pairs and on the one-CTA kernel (whose tiles are then visited in bands,
    the banded tile decoder);
  * the one-CTA square at n = 2048 (16 row blocks, plain row order);
  * wide and tall Grams with long K (m = 2n) at n = 2304 and 4096.

Whole circuits against the FP64 evaluation of the same circuit
(oracle.circuit, one FP16 rounding per iteration), with the tolerance rule of
test_gpu_circuit.py: relative Frobenius <= 5e-3 unless the FP32-vs-FP64
oracle distance (the floor, measured on the same input) exceeds 2.5e-3, then
1.5 x the floor; singular-value endpoints within 1e-3 (2e-3 for PS3 tables).
Every case prints its error, floor and tolerance (pytest -rP shows them):
  * X = U diag(s) V^T with s log-uniform on [1e-3, 1],
    n = 2048, alpha in {1, 2}, PS2-55 and PS3-55, FP16 input;
  * BASELINE config 3 (NanoGPT batch, PS3-55), one Qwen3-0.6B layer
    (config 4, PS2-55) and one Gemma-3-1B layer (config 5, PS3-55) through
    the grouped call, each matrix of the call checked against its own oracle
    evaluation (a sample of the NanoGPT batch: first, middle, last of a bank).
"""

import pytest
import torch

from oracle import circuit as oc
from polar_switch import coefficients
from tests._util import assert_fp16_close, log_uniform_matrix, seeded

pytestmark = pytest.mark.gpu

REL_FRO_TOL = 5e-3
SIGMA_TOL = 1e-3
SIGMA_TOL_PS3 = 2e-3


@pytest.fixture(params=["default", "onecta"])
def kernel_mode(request):
    """Run a test on the default kernel (CTA pairs), then on the one-CTA kernel,
    whose symmetric tiles above 16 row blocks go through the banded decoder."""
    from polar_switch import _native as nat
    if request.param == "default":
        yield request.param
        return
    prev = nat.set_cta_pairs(0)
    try:
        yield request.param
    finally:
        nat.set_cta_pairs(prev)


def _sym_random(n, L, seed):
    """Bit-symmetric FP16 matrices with entries of variance 1/n."""
    G = seeded((L, n, n), seed)
    return ((G + G.mT) / (2 * n) ** 0.5).half()


@pytest.mark.parametrize("L,n,inplace", [(1, 2048, False), (1, 2304, False), (1, 2304, True),
                                         (1, 4096, False), (2, 2176, True)])
def test_square_banded_and_long(cuda_device, kernel_mode, L, n, inplace):
    from polar_switch import cuda_ops
    A = _sym_random(n, L, 900 + n)
    C = _sym_random(n, L, 901 + n)
    alpha, beta, diag = 1.75, -0.6, 0.37
    Ad, Cd = A.to(cuda_device), C.to(cuda_device)
    out = Cd if inplace else torch.empty_like(Ad)
    cuda_ops.square(Ad, Cd, out, alpha, beta, diag)
    ref = oc.square(A, C, alpha, beta, diag)
    Af = A.float()
    terms = abs(alpha) * (Af @ Af.mT).abs() + abs(beta) * C.float().abs() + abs(diag)
    assert_fp16_close(out, ref, what=f"square {L}x{n} inplace={inplace} ({kernel_mode})",
                      terms=terms, k=n)
    o = out.cpu()
    assert torch.equal(o, o.mT)


@pytest.mark.parametrize("L,rows,cols", [(1, 2304, 4608), (1, 4608, 2304), (1, 4096, 8192),
                                         (1, 8192, 4096), (2, 2200, 2304)])
def test_gram_long_k(cuda_device, kernel_mode, L, rows, cols):
    from polar_switch import cuda_ops
    X = oc.normalize(seeded((L, rows, cols), 910 + rows + cols), 1e-7)
    tall = rows > cols
    n = min(rows, cols)
    out = torch.empty(L, n, n, dtype=torch.float16, device=cuda_device)
    cuda_ops.gram(X.to(cuda_device), tall, out)
    ref = oc.gram(X, tall)
    assert_fp16_close(out, ref, what=f"gram {L}x{rows}x{cols} ({kernel_mode})")
    o = out.cpu()
    assert torch.equal(o, o.mT)


@pytest.mark.parametrize("L,rows,cols", [(1, 2048, 4096), (1, 4608, 2304)])
def test_apply_large(cuda_device, L, rows, cols):
    from polar_switch import cuda_ops
    X = oc.normalize(seeded((L, rows, cols), 920 + rows), 1e-7)
    n = min(rows, cols)
    B = _sym_random(n, L, 921 + n)
    tall = rows > cols
    out = cuda_ops.apply(X.to(cuda_device), B.to(cuda_device), tall, 0.0)
    ref = oc.apply(X, B, tall, 0.0)
    assert_fp16_close(out, ref, what=f"apply {L}x{rows}x{cols}")


def _parity(name, got, X, table, method):
    """Compare one matrix's result with the FP64 oracle; print and return the figures."""
    ref64 = oc.run_circuit(X, table, acc=torch.float64)
    ref32 = oc.run_circuit(X, table, acc=torch.float32)
    err = oc.relative_frobenius(got, ref64)
    floor = oc.relative_frobenius(ref32, ref64)
    rel_tol = REL_FRO_TOL if floor <= REL_FRO_TOL / 2 else 1.5 * floor
    lo, hi = oc.singular_interval(got)
    rlo, rhi = oc.singular_interval(ref64)
    stol = SIGMA_TOL_PS3 if method.startswith("PS3") or min(X.shape[-2:]) < 512 else SIGMA_TOL
    line = (f"PARITY {name} {method} {tuple(X.shape)}: rel-Fro {err:.3e} floor {floor:.3e} tol {rel_tol:.3e}"
            f"{' (relaxed)' if rel_tol > REL_FRO_TOL else ''}; sigma [{lo:.5f}, {hi:.5f}] vs "
            f"[{rlo:.5f}, {rhi:.5f}] tol {stol:.0e}")
    print(line)
    assert err <= rel_tol, line
    assert abs(lo - rlo) <= stol and abs(hi - rhi) <= stol, line
    return err, floor


@pytest.mark.parametrize("method", ["PS2_55", "PS3_55"])
@pytest.mark.parametrize("alpha", [1, 2])
def test_config2_log_uniform_n2048(cuda_device, method, alpha):
    from polar_switch import make_polynomial_orthogonalizer
    n = 2048
    X = log_uniform_matrix(n, alpha * n, seed=2000 + alpha).half()
    polar = make_polynomial_orthogonalizer(method)
    got = polar(X.to(cuda_device)).cpu()
    assert got.dtype == torch.float16 and got.shape == X.shape
    _parity("config2", got, X, getattr(coefficients, method), method)


def _grouped_parity(name, banks, method, device, sample=None):
    from polar_switch import make_polynomial_orthogonalizer
    polar = make_polynomial_orthogonalizer(method)
    outs = polar.grouped([b.to(device) for b in banks])
    table = getattr(coefficients, method)
    for bank, out in zip(banks, outs):
        assert out.shape == bank.shape and out.dtype == bank.dtype
        L = bank.shape[0]
        idx = sorted({0, L // 2, L - 1}) if sample else range(L)
        for i in idx:
            _parity(f"{name}[{tuple(bank.shape)}][{i}]", out[i].cpu(), bank[i], table, method)


def test_config3_nanogpt_batch_grouped(cuda_device):
    """48 x 768^2 + 12 x 768x3072 + 12 x 3072x768, FP32 N(0, 0.02^2), PS3-55."""
    g = torch.Generator().manual_seed(3)
    banks = [torch.randn(L, r, c, generator=g) * 0.02 for L, r, c in
             ((48, 768, 768), (12, 768, 3072), (12, 3072, 768))]
    _grouped_parity("config3", banks, "PS3_55", cuda_device, sample=True)


def test_config4_qwen_layer_grouped(cuda_device):
    """One Qwen3-0.6B layer: q 2048x1024, k/v 1024^2, o 1024x2048, gate/up 3072x1024,
    down 1024x3072, FP32 N(0, 1), PS2-55."""
    g = torch.Generator().manual_seed(4)
    banks = [torch.randn(L, r, c, generator=g) for L, r, c in
             ((1, 2048, 1024), (2, 1024, 1024), (1, 1024, 2048), (2, 3072, 1024), (1, 1024, 3072))]
    _grouped_parity("config4", banks, "PS2_55", cuda_device)


def test_config5_gemma_layer_grouped(cuda_device):
    """One Gemma-3-1B layer: q 1024x1152, k/v 256x1152, o 1152x1024, gate/up
    6912x1152, down 1152x6912, FP32 N(0, 1), PS3-55."""
    g = torch.Generator().manual_seed(5)
    banks = [torch.randn(L, r, c, generator=g) for L, r, c in
             ((1, 1024, 1152), (2, 256, 1152), (1, 1152, 1024), (2, 6912, 1152), (1, 1152, 6912))]
    _grouped_parity("config5", banks, "PS3_55", cuda_device)
