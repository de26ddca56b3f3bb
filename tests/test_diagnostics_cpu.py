"""Update telemetry on CPU: the Lanczos core (it runs on any device, given
the Gram), the log format, and the product refusing CPU tensors. The GPU
paths (ps_update_stats, the tensor-core Gram) are in test_gpu_diagnostics."""

import gzip
import json

import pytest
import torch

from polar_switch import diagnostics as dg


def _matrices(shapes_seed, B, m, n, spread=1.0):
    g = torch.Generator().manual_seed(shapes_seed)
    return torch.randn(B, m, n, generator=g, dtype=torch.float64) * spread


def _exact(A):
    return torch.linalg.matrix_norm(A.double(), ord=2)


@pytest.mark.parametrize("B,m,n,probes", [(3, 60, 40, 4), (2, 48, 48, 1), (4, 100, 24, 2)])
def test_lanczos_gram_matches_exact_norms(B, m, n, probes):
    A = _matrices(1, B, m, n)
    G = (A.mT @ A).float()
    est, info = dg.lanczos_gram(G, probes=probes)
    assert torch.allclose(est.double(), _exact(A), rtol=1e-4)
    assert info["converged"].all() and info["convergence_assessed"].all()
    assert info["iterations"] >= 32 and info["iterations"] % 16 == 0
    assert (info["ritz_residual"] <= 1e-3).all()
    assert info["projection_fp64_retries"] == 0


def test_lanczos_gram_clustered_spectrum():
    """Nearly orthogonal matrices (all singular values in [0.87, 1.11], like
    the orthogonalizers' outputs): the estimate stays within rtol of the top
    singular value and below it."""
    g = torch.Generator().manual_seed(5)
    Q, _ = torch.linalg.qr(torch.randn(3, 80, 64, generator=g, dtype=torch.float64))
    s = 0.87 + 0.24 * torch.rand(3, 64, generator=g, dtype=torch.float64)
    V, _ = torch.linalg.qr(torch.randn(3, 64, 64, generator=g, dtype=torch.float64))
    A = Q @ torch.diag_embed(s) @ V.mT
    est, _ = dg.lanczos_gram((A.mT @ A).float(), probes=1, max_iter=64)
    exact = _exact(A)
    assert ((est.double() - exact).abs() / exact <= 1e-3).all()
    assert (est.double() <= exact * (1 + 1e-5)).all()


def test_lanczos_gram_zero_matrix_and_short_runs():
    A = _matrices(2, 3, 30, 20)
    A[1] = 0
    est, info = dg.lanczos_gram((A.mT @ A).float(), max_iter=16)
    assert est[1] == 0 and info["converged"][1] and info["convergence_assessed"][1]
    # 16 iterations: convergence is tested once, against no earlier estimate
    assert not info["convergence_assessed"][0] and torch.isnan(info["relative_change"][0])
    assert info["iterations"] == 16
    assert torch.allclose(est[0].double(), _exact(A[0]), rtol=1e-4)


def test_lanczos_gram_ignores_zero_padding():
    A = _matrices(3, 2, 50, 30)
    G = (A.mT @ A).float()
    Gp = torch.zeros(2, 40, 40)
    Gp[:, :30, :30] = G
    est, _ = dg.lanczos_gram(G)
    estp, _ = dg.lanczos_gram(Gp, n_valid=30)
    assert torch.allclose(est, estp, rtol=1e-5)


def test_lanczos_gram_rejects_bad_arguments():
    with pytest.raises(ValueError):
        dg.lanczos_gram(torch.zeros(2, 3, 4))
    with pytest.raises(ValueError):
        dg.lanczos_gram(torch.zeros(2, 4, 4), max_iter=8)
    with pytest.raises(ValueError):
        dg.lanczos_gram(torch.zeros(2, 4, 4), rtol=0)


def _cpu_stats(m):
    nan = torch.isnan(m).sum(dim=(-2, -1))
    inf = torch.isinf(m).sum(dim=(-2, -1))
    return nan, inf, m.abs().amax(dim=(-2, -1)).float()


def _cpu_estimator(m, probes, max_iter, rtol):
    a = m.double()
    G = (a.mT @ a if a.shape[-2] >= a.shape[-1] else a @ a.mT).float()
    return dg.lanczos_gram(G, probes=probes, max_iter=max_iter, rtol=rtol)


def _read(path):
    with gzip.open(path, "rt") as f:
        return [json.loads(line) for line in f]


def test_norm_log_records_in_the_reference_format(tmp_path):
    log = dg.NormLog(tmp_path, rank=3, method="PS2_55", stats=_cpu_stats, estimator=_cpu_estimator)
    X = _matrices(4, 4, 24, 40).float()
    X[1, 2, 3] = float("nan")
    X[2, 0, 0] = float("inf")
    log.step = 7
    log.record("mlp", X, matrix_start=8, execution={"backend": "b200"}, matrix_names=["a", "b", "c", "d"])
    log.close()
    assert log.path.name.startswith("rank-0003-") and log.path.name.endswith(".jsonl.gz")
    meta, rec = _read(log.path)
    assert meta == dict(event="metadata", format="polar-output-norm-v2", method="PS2_55", rank=3,
                        estimator="Lanczos", probes=1, max_iter=64, rtol=0.001, estimate_only=True,
                        stage="post_orthogonalization_before_optimizer_scaling",
                        step_index="zero-based, excludes warmup")
    assert list(rec) == ["event", "step", "label", "matrix_start", "matrix_names", "shape", "dtype",
                         "requested", "execution", "spectral_norm", "max_abs", "nan_count", "inf_count",
                         "converged", "convergence_assessed", "ritz_residual", "relative_change",
                         "iterations", "projection_fp64_retries", "estimator_error"]
    assert rec["event"] == "orthogonalization" and rec["step"] == 7 and rec["label"] == "mlp"
    assert rec["matrix_start"] == 8 and rec["shape"] == [4, 24, 40] and rec["dtype"] == "torch.float32"
    assert rec["nan_count"] == [0, 1, 0, 0] and rec["inf_count"] == [0, 0, 1, 0]
    assert rec["spectral_norm"][1] is None and rec["spectral_norm"][2] is None
    assert rec["max_abs"][1] is None and rec["max_abs"][2] is None  # NaN / inf are not JSON numbers
    for i in (0, 3):
        exact = float(_exact(X[i].double()))
        assert abs(rec["spectral_norm"][i] - exact) <= 1e-4 * exact
        assert rec["max_abs"][i] == float(X[i].abs().max())
        assert rec["converged"][i] and rec["convergence_assessed"][i]
    assert rec["converged"][1] is False and rec["iterations"] >= 32 and rec["estimator_error"] is None


def test_norm_log_keeps_estimator_failures(tmp_path):
    def failing(m, probes, max_iter, rtol):
        raise torch.linalg.LinAlgError("no convergence")
    log = dg.NormLog(tmp_path, rank=0, method="PS3_55", stats=_cpu_stats, estimator=failing)
    log.record("attn", _matrices(6, 2, 16, 16).float())
    log.close()
    _, rec = _read(log.path)
    assert rec["estimator_error"] == "no convergence" and rec["spectral_norm"] == [None, None]
    assert rec["iterations"] == 0


def test_gpu_telemetry_refuses_cpu_tensors(tmp_path):
    from polar_switch import cuda_ops
    X = torch.randn(2, 16, 24)
    with pytest.raises(NotImplementedError):
        cuda_ops.update_stats(X)
    with pytest.raises(NotImplementedError):
        dg.spectral_norm(X)
    with pytest.raises(ValueError):
        dg.spectral_norm(torch.randn(16, 24))
    log = dg.NormLog(tmp_path, rank=0, method="PS2_55")
    with pytest.raises(NotImplementedError):
        log.record("x", X)
    log.close()
