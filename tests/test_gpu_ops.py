"""Parity of each B200 kernel (gram, square, sym_product, apply, normalize,
add_diag) with the CPU oracle on the same seeded inputs.

One contraction accumulated in FP32 and rounded once to FP16 can differ from
another FP32 accumulation only by rounding flips, so the bar is: every element
within 1 FP16 ulp of the oracle, and at most a few percent of elements not
bit-identical.
"""

import pytest
import torch

from oracle import circuit as oc
from tests._util import assert_fp16_close, seeded

pytestmark = pytest.mark.gpu


def _sym(n, L, seed):
    """A symmetric FP16 matrix with Gram-like entries (normalised X @ X.T)."""
    X = oc.normalize(seeded((L, n, 2 * n), seed), 1e-7)
    return oc.gram(X, False)


@pytest.mark.parametrize("L,rows,cols", [(2, 128, 256), (1, 256, 512), (3, 96, 200),
                                         (1, 384, 1024), (2, 8, 64), (1, 520, 136),
                                         (2, 256, 128), (1, 1024, 1152)])
def test_gram(cuda_device, L, rows, cols):
    from polar_switch import cuda_ops
    X = oc.normalize(seeded((L, rows, cols), 1 + rows + cols), 1e-7)
    tall = rows > cols
    n = min(rows, cols)
    out = torch.empty(L, n, n, dtype=torch.float16, device=cuda_device)
    cuda_ops.gram(X.to(cuda_device), tall, out)
    ref = oc.gram(X, tall)
    assert_fp16_close(out, ref, what=f"gram {L}x{rows}x{cols}")
    # symmetric by construction (mirrored store)
    o = out.cpu()
    assert torch.equal(o, o.mT)


@pytest.mark.parametrize("L,n", [(1, 128), (2, 256), (1, 384), (3, 136), (2, 8), (1, 1152)])
@pytest.mark.parametrize("inplace", [False, True])
def test_square(cuda_device, L, n, inplace):
    from polar_switch import cuda_ops
    A = _sym(n, L, 10 + n)
    C = _sym(n, L, 20 + n)
    alpha, beta, diag = 1.75, -0.6, 0.37
    Ad, Cd = A.to(cuda_device), C.to(cuda_device)
    out = Cd if inplace else torch.empty_like(Ad)
    cuda_ops.square(Ad, Cd, out, alpha, beta, diag)
    ref = oc.square(A, C, alpha, beta, diag)
    assert_fp16_close(out, ref, what=f"square {L}x{n} inplace={inplace}")


def test_square_ps2_coefficients(cuda_device):
    """The large coefficients of PS2-55 (a=164.08, b=49.58) on a realistic buffer."""
    from polar_switch import cuda_ops
    A = _sym(256, 2, 7)
    ref = oc.square(A, A, 164.07644513428048, 49.58061223879703, 0.000500089059050944)
    Ad = A.to(cuda_device)
    out = torch.empty_like(Ad)
    cuda_ops.square(Ad, Ad, out, 164.07644513428048, 49.58061223879703, 0.000500089059050944)
    assert_fp16_close(out, ref, what="square PS2-55 step 2")


@pytest.mark.parametrize("L,n", [(1, 256), (2, 136)])
def test_sym_product(cuda_device, L, n):
    from polar_switch import cuda_ops
    P = _sym(n, L, 30 + n)
    Q = _sym(n, L, 40 + n)
    C = _sym(n, L, 50 + n)
    out = cuda_ops.sym_product(P.to(cuda_device), Q.to(cuda_device), C.to(cuda_device),
                               alpha=0.8, beta=1.3, diag=-0.25)
    ref = oc.sym_product(P, Q, C, 0.8, 1.3, -0.25)
    assert_fp16_close(out, ref, what=f"sym_product {L}x{n}")


@pytest.mark.parametrize("L,rows,cols", [(2, 128, 256), (1, 256, 1024), (3, 96, 200), (1, 136, 520),
                                         (2, 256, 128), (1, 1024, 384), (2, 200, 96)])
@pytest.mark.parametrize("residual", [0.0, 3.4445])
def test_apply(cuda_device, L, rows, cols, residual):
    from polar_switch import cuda_ops
    X = oc.normalize(seeded((L, rows, cols), 60 + rows), 1e-7)
    n = min(rows, cols)
    B = _sym(n, L, 70 + n)
    tall = rows > cols
    out = cuda_ops.apply(X.to(cuda_device), B.to(cuda_device), tall, residual)
    ref = oc.apply(X, B, tall, residual)
    assert_fp16_close(out, ref, what=f"apply {L}x{rows}x{cols} residual={residual}")


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_apply_widened_output(cuda_device, out_dtype):
    from polar_switch import cuda_ops
    X = oc.normalize(seeded((2, 256, 512), 5), 1e-7)
    B = _sym(256, 2, 6)
    got = cuda_ops.apply(X.to(cuda_device), B.to(cuda_device), False, 0.0, out_dtype=out_dtype)
    ref16 = oc.apply(X, B, False, 0.0)
    assert got.dtype == out_dtype
    if out_dtype == torch.float32:
        # the FP32 output is exactly the FP16 result widened
        assert torch.equal(got.cpu(), got.cpu().half().float())
        assert_fp16_close(got.half(), ref16, what="apply -> float32")
    else:
        # BF16 output = bf16(fp16 result): equal to the oracle's converted value
        # up to one BF16 rounding flip, or one FP16 flip carried through (near 0)
        from tests._util import fp16_ulp
        g = got.float().cpu()
        r = ref16.to(torch.bfloat16).float()
        ulp = torch.pow(2.0, torch.floor(torch.log2(r.abs().clamp_min(2.0 ** -126))) - 7)
        assert ((g - r).abs() <= ulp + fp16_ulp(ref16)).all()
        assert float(((g - r) != 0).float().mean()) < 0.01


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16, torch.float64])
@pytest.mark.parametrize("shape", [(3, 64, 96), (1, 1000, 24), (2, 7, 5), (2, 1024, 3072), (5, 200, 1152)])
def test_normalize(cuda_device, dtype, shape):
    from polar_switch import cuda_ops
    X = seeded(shape, 80, dtype=dtype, scale=3.0)
    got = cuda_ops.normalize(X.to(cuda_device), 1e-7)
    ref = oc.normalize(X, 1e-7)
    assert_fp16_close(got, ref, max_ulps=1, max_mismatch=0.01, what=f"normalize {dtype} {shape}")


@pytest.mark.parametrize("dtype,shape", [(torch.float32, (3, 1024, 3072)), (torch.float16, (4, 1152, 1024)),
                                         (torch.bfloat16, (3, 384, 520)), (torch.float64, (2, 768, 768)),
                                         (torch.float32, (2, 4096, 4096))])
def test_normalize_is_batch_independent(cuda_device, dtype, shape):
    """Contiguous matrices are reduced over fixed chunks, so a slice of a batch
    normalises to exactly the bits of the same matrices in the whole batch
    (the sharded Muon step relies on this to match a single process)."""
    from polar_switch import cuda_ops
    X = seeded(shape, 82, dtype=dtype, scale=2.0).to(cuda_device)
    whole = cuda_ops.normalize(X, 1e-7)
    part = cuda_ops.normalize(X[1:], 1e-7)
    one = cuda_ops.normalize(X[-1:], 1e-7)
    assert torch.equal(part, whole[1:])
    assert torch.equal(one, whole[-1:])
    assert_fp16_close(whole.cpu(), oc.normalize(X.cpu(), 1e-7), max_ulps=1, max_mismatch=0.01,
                      what=f"normalize {dtype} {shape}")


def test_normalize_strided(cuda_device):
    from polar_switch import cuda_ops
    X = seeded((4, 96, 64), 81)
    Xt = X.to(cuda_device).mT  # non-contiguous (4, 64, 96)
    got = cuda_ops.normalize(Xt, 1e-7)
    ref = oc.normalize(X.mT, 1e-7)
    assert_fp16_close(got, ref, what="normalize transposed view")


def test_add_diag(cuda_device):
    from polar_switch import cuda_ops
    Z = _sym(64, 3, 90)
    got = cuda_ops.add_diag(Z.to(cuda_device), 2.365477637327074)
    ref = oc.add_diag(Z, 2.365477637327074)
    assert torch.equal(got.cpu(), ref)


@pytest.mark.parametrize("L,rows,cols", [(2, 256, 128), (2, 128, 384), (1, 200, 136)])
def test_apply_general_b_is_exact_product(cuda_device, L, rows, cols):
    """apply multiplies by B exactly as stored (B @ X or X @ B), symmetric or not."""
    from polar_switch import cuda_ops
    X = oc.normalize(seeded((L, rows, cols), 90 + rows), 1e-7)
    n = min(rows, cols)
    B = (seeded((L, n, n), 91 + n) / n ** 0.5).half()  # not symmetric
    tall = rows > cols
    out = cuda_ops.apply(X.to(cuda_device), B.to(cuda_device), tall, 0.5)
    ref = oc.apply(X, B, tall, 0.5)
    assert_fp16_close(out, ref, what=f"apply general B {L}x{rows}x{cols}")


def test_sym_product_is_p_at_q(cuda_device):
    """Upper tiles are P @ Q with Q read as stored (not Q^T), mirrored below."""
    from polar_switch import cuda_ops
    P = _sym(256, 2, 92)
    Q = (seeded((2, 256, 256), 93) / 16).half()  # deliberately not symmetric
    out = cuda_ops.sym_product(P.to(cuda_device), Q.to(cuda_device), None, alpha=1.0, beta=0.0)
    ref = oc.sym_product(P, Q, None, 1.0, 0.0)
    assert_fp16_close(out, ref, what="sym_product P@Q")


@pytest.mark.parametrize("shape,dtype", [((3, 1024, 3072), torch.float32), ((2, 384, 128), torch.bfloat16),
                                         ((4, 200, 72), torch.float16)])
def test_sumsq_and_scale_cast_compose_to_normalize(cuda_device, shape, dtype):
    """The two pieces of the split-matrix normalisation give ps_normalize's
    bits when the sums are not split; without sums scale_cast is .half()."""
    from polar_switch import cuda_ops
    X = seeded(shape, 97, dtype=dtype, scale=2.0).to(cuda_device)
    sums = cuda_ops.sumsq(X)
    assert sums.dtype == torch.float64 and sums.shape == (shape[0],)
    ref = X.double().pow(2).sum(dim=(-2, -1))
    assert torch.allclose(sums, ref, rtol=1e-5)
    assert torch.equal(cuda_ops.scale_cast(X, sums, 1e-7), cuda_ops.normalize(X, 1e-7))
    G = torch.randn(2, 256, 256, device=cuda_device)
    assert torch.equal(cuda_ops.scale_cast(G, None, 0.0), G.half())
    part = X[..., : shape[-1] // 2]  # strided view, as a split matrix's part
    assert torch.allclose(cuda_ops.sumsq(part), part.double().pow(2).sum(dim=(-2, -1)), rtol=1e-5)


@pytest.mark.parametrize("shape", [(2, 256, 768), (1, 640, 128), (3, 136, 136)])
def test_gram_f32_is_the_unrounded_gram(cuda_device, shape):
    from polar_switch import cuda_ops
    X = oc.normalize(seeded(shape, 98), 1e-7)
    got = cuda_ops.gram_f32(X.to(cuda_device)).cpu()
    Xa = X.double()
    ref = Xa.mT @ Xa if shape[-2] > shape[-1] else Xa @ Xa.mT
    assert got.dtype == torch.float32
    # tensor-core FP32 accumulation: well inside one FP16 ulp (4.9e-4 relative)
    assert float((got.double() - ref).norm() / ref.norm()) < 5e-4
    assert torch.equal(got, got.mT)  # both triangles from the same products
    # rounded once, it is the FP16 Gram of the symmetric kernel to within one ulp
    fp16 = torch.empty(shape[0], min(shape[1:]), min(shape[1:]), device=cuda_device, dtype=torch.float16)
    cuda_ops.gram(X.to(cuda_device), shape[-2] > shape[-1], fp16)
    assert_fp16_close(got.half(), fp16.cpu(), max_ulps=1, max_mismatch=0.02, what=f"gram_f32 {shape}")
