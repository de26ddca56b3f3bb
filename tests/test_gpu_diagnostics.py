"""Update telemetry on the GPU: ps_update_stats against torch's three passes
(exact: counts and maxima do not depend on order), the spectral-norm
estimator (tensor-core Gram + Lanczos) against the exact spectral norm, and
NormLog end to end."""

import gzip
import json

import pytest
import torch

from polar_switch import cuda_ops, diagnostics as dg, make_polynomial_orthogonalizer
from tests._util import seeded

pytestmark = pytest.mark.gpu


def _torch_stats(m):
    return (torch.isnan(m).sum(dim=(-2, -1)), torch.isinf(m).sum(dim=(-2, -1)),
            m.abs().amax(dim=(-2, -1)).float())


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(5, 64, 96), (3, 17, 33), (2, 1024, 3072), (1, 1, 7), (70, 8, 8)])
def test_update_stats_match_torch(cuda_device, dtype, shape):
    X = seeded(shape, 700).to(dtype).to(cuda_device)
    L = shape[0]
    X.view(L, -1)[0, -1] = float("nan")             # last element: the unvectorised tail when E % 8
    X.view(L, -1)[L - 1, 0] = float("-inf")
    if L > 2:
        X[1].fill_(float("nan"))                    # a matrix with no number at all
        X[2].view(-1)[::3] = float("inf")
        X[2].view(-1)[1] = -0.0
    got = cuda_ops.update_stats(X)
    exp = _torch_stats(X)
    assert torch.equal(got[0], exp[0]) and torch.equal(got[1], exp[1])
    assert torch.equal(torch.isnan(got[2]), torch.isnan(exp[2]))
    finite = ~torch.isnan(exp[2])
    assert torch.equal(got[2][finite], exp[2][finite])


def test_update_stats_offset_view_and_batch_shape(cuda_device):
    """A view that does not start on a 16-byte boundary takes the scalar loop;
    leading batch dimensions are kept."""
    base = seeded((4 * 40 * 24 + 1,), 701).half().to(cuda_device)
    X = base[1:].view(2, 2, 40, 24)
    X[1, 0, 3, 5] = float("inf")
    nan, inf, amax = cuda_ops.update_stats(X)
    assert nan.shape == (2, 2) and inf.tolist() == [[0, 0], [1, 0]]
    assert torch.equal(amax, X.abs().amax(dim=(-2, -1)).float())


@pytest.mark.parametrize("dtype,shape", [(torch.bfloat16, (4, 256, 512)), (torch.float32, (2, 1000, 296)),
                                         (torch.float16, (3, 130, 66)), (torch.float32, (2, 70, 65))])
def test_spectral_norm_matches_exact(cuda_device, dtype, shape):
    X = (seeded(shape, 702) * 3.0).to(dtype).to(cuda_device)
    est, info = dg.spectral_norm(X)
    exact = torch.linalg.matrix_norm(X.double(), ord=2)
    rel = ((est.double() - exact).abs() / exact)
    assert (rel <= 2e-3).all(), rel
    assert info["iterations"] >= 32 and info["projection_fp64_retries"] == 0


def test_spectral_norm_of_orthogonalized_updates(cuda_device):
    """The use the log is for: outputs of PS2_55 (singular values in about
    [0.87, 1.11]), estimated with the log's settings."""
    X = seeded((6, 384, 768), 703).to(cuda_device)
    U = make_polynomial_orthogonalizer("PS2_55")(X)
    est, _ = dg.spectral_norm(U, probes=1, max_iter=64, rtol=1e-3)
    exact = torch.linalg.matrix_norm(U.double(), ord=2)
    assert ((est.double() - exact).abs() / exact <= 5e-3).all()


def test_spectral_norm_zero_matrix(cuda_device):
    X = torch.zeros(2, 64, 32, device=cuda_device, dtype=torch.float16)
    X[1] = seeded((64, 32), 704).half().to(cuda_device)
    est, info = dg.spectral_norm(X)
    assert est[0] == 0 and info["converged"][0]
    exact = torch.linalg.matrix_norm(X[1].double(), ord=2)
    assert abs(float(est[1]) - float(exact)) <= 2e-3 * float(exact)


def test_norm_log_end_to_end(cuda_device, tmp_path):
    log = dg.NormLog(tmp_path, rank=1, method="PS2_55")
    U = make_polynomial_orthogonalizer("PS2_55")(seeded((4, 256, 128), 705).to(cuda_device))
    U[2, 0, 0] = float("nan")
    log.record("mlp", U, matrix_start=4)
    log.close()
    with gzip.open(log.path, "rt") as f:
        meta, rec = [json.loads(line) for line in f]
    assert meta["format"] == "polar-output-norm-v2" and rec["nan_count"] == [0, 0, 1, 0]
    assert rec["spectral_norm"][2] is None and rec["max_abs"][2] is None
    for i in (0, 1, 3):
        exact = float(torch.linalg.matrix_norm(U[i].double(), ord=2))
        assert abs(rec["spectral_norm"][i] - exact) <= 5e-3 * exact
        assert rec["max_abs"][i] == float(U[i].abs().max())
