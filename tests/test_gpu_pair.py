"""The CTA-pair GEMM kernel (tcgen05 cta_group::2, 256 x 256 tiles) against
the one-CTA kernel and the oracle, on shapes that exercise its tile edges:
odd numbers of 128-row blocks (the last column pair and row pair half out of
range), partial blocks, tall and wide operands, and batches. Sizes that are
multiples of 64 load each 128-wide K stage with one TMA over a 4-D chunked
view (1088 = 17 x 64: the last stage half out of range), other sizes with
two or four 3-D boxes; both fill the same shared-memory layout."""

import pytest
import torch

from oracle import circuit as oc
from tests._util import assert_fp16_close, seeded

pytestmark = pytest.mark.gpu


def _sym(n, L, seed):
    X = oc.normalize(seeded((L, n, 2 * n), seed), 1e-7)
    return oc.gram(X, False)


def _both(fn):
    """Run fn() with the pair kernel and with the one-CTA kernel."""
    from polar_switch import _native as nat
    prev = nat.set_cta_pairs(True)
    try:
        a = fn().cpu()
        nat.set_cta_pairs(False)
        b = fn().cpu()
    finally:
        nat.set_cta_pairs(prev)
    return a, b


@pytest.mark.parametrize("L,n", [(1, 128), (2, 256), (1, 384), (3, 136), (1, 1152), (2, 640), (1, 8),
                                 (1, 1088), (2, 192)])
def test_square_pair_vs_single(cuda_device, L, n):
    from polar_switch import cuda_ops
    A = _sym(n, L, 300 + n).to(cuda_device)
    C = _sym(n, L, 301 + n).to(cuda_device)

    def run():
        out = torch.empty_like(A)
        return cuda_ops.square(A, C, out, 1.3, -0.4, 0.2)

    pair, single = _both(run)
    ref = oc.square(A.cpu(), C.cpu(), 1.3, -0.4, 0.2)
    assert_fp16_close(pair, ref, what=f"pair square {L}x{n}")
    assert_fp16_close(pair, single, what=f"pair vs single square {L}x{n}")
    assert torch.equal(pair, pair.mT)


@pytest.mark.parametrize("L,rows,cols", [(2, 384, 1024), (1, 1152, 1000), (3, 520, 136), (1, 96, 200),
                                         (1, 1088, 2112), (2, 2112, 1088), (1, 320, 192)])
def test_gram_pair_vs_single(cuda_device, L, rows, cols):
    from polar_switch import cuda_ops
    X = oc.normalize(seeded((L, rows, cols), 310 + rows), 1e-7).to(cuda_device)
    tall = rows > cols
    n = min(rows, cols)

    def run():
        out = torch.empty(L, n, n, device=cuda_device, dtype=torch.float16)
        return cuda_ops.gram(X, tall, out)

    pair, single = _both(run)
    assert_fp16_close(pair, oc.gram(X.cpu(), tall), what="pair gram")
    assert_fp16_close(pair, single, what="pair vs single gram")


@pytest.mark.parametrize("L,rows,cols", [(2, 256, 1024), (1, 1152, 384), (3, 200, 96), (1, 136, 520),
                                         (2, 640, 2048), (1, 1088, 2112), (1, 2112, 1088)])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
def test_apply_pair_vs_single(cuda_device, L, rows, cols, out_dtype):
    from polar_switch import cuda_ops
    X = oc.normalize(seeded((L, rows, cols), 320 + rows), 1e-7).to(cuda_device)
    n = min(rows, cols)
    B = _sym(n, L, 321 + n).to(cuda_device)
    tall = rows > cols

    def run():
        return cuda_ops.apply(X, B, tall, 2.5, out_dtype=out_dtype)

    pair, single = _both(run)
    ref = oc.apply(X.cpu(), B.cpu(), tall, 2.5)
    assert_fp16_close(pair.half(), ref, what="pair apply")
    assert_fp16_close(pair.half(), single.half(), what="pair vs single apply")


def test_sym_product_pair(cuda_device):
    from polar_switch import cuda_ops
    P = _sym(384, 2, 330).to(cuda_device)
    Q = (seeded((2, 384, 384), 331) / 20).half().to(cuda_device)  # not symmetric: exact P @ Q
    pair, single = _both(lambda: cuda_ops.sym_product(P, Q, None, alpha=1.0, beta=0.0))
    assert_fp16_close(pair, oc.sym_product(P.cpu(), Q.cpu(), None, 1.0, 0.0), what="pair P@Q")
    assert_fp16_close(pair, single, what="pair vs single P@Q")


def test_circuit_pair_vs_single(cuda_device):
    from polar_switch import make_polynomial_orthogonalizer
    X = seeded((3, 384, 1152), 340).to(cuda_device)
    polar = make_polynomial_orthogonalizer("PS3_55")
    pair, single = _both(lambda: polar(X))
    assert oc.relative_frobenius(pair, single) < 2e-3


@pytest.mark.parametrize("method,shape", [("PS2_55", (2, 384, 1152)), ("PS3_55", (1152, 640)),
                                          ("POLAR_EXPRESS", (3, 256, 384)), ("PS2_55", (1, 200, 72)),
                                          ("PS3_55", (1, 1088, 2176))])
def test_triangle_storage_circuit_is_bit_identical(cuda_device, method, shape):
    """Inside a circuit the square buffers are kept as upper-triangle blocks and
    read back transposed; the result must equal, bit for bit, the op-by-op
    evaluation through the public kernels that store full mirrored buffers."""
    import polar_switch
    from polar_switch import coefficients, cuda_ops
    X = seeded(shape, 350).to(cuda_device)
    table = getattr(coefficients, method)
    fused = polar_switch.make_polynomial_orthogonalizer(method)(X)
    buffers = polar_switch.validate_table(table, 1e-7)
    op_by_op = polar_switch._run(X, table, cuda_ops, 1e-7, buffers).to(X.dtype)
    assert torch.equal(fused, op_by_op)
