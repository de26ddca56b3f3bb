"""torch.compile(fullgraph=True) over the orthogonalizers and over the
op-by-op evaluator with the operator backend: no graph breaks, and the
compiled results equal the eager ones bit for bit."""

import pytest
import torch

import polar_switch
from polar_switch import coefficients, cuda_ops, make_polynomial_orthogonalizer, torch_ops
from tests._util import seeded

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("method,shape", [("PS3_55", (2, 256, 512)), ("PS2_55", (384, 128)),
                                          ("GNS", (2, 128, 384))])
def test_orthogonalizer_under_torch_compile(cuda_device, method, shape):
    polar = make_polynomial_orthogonalizer(method)
    X = seeded(shape, 95).to(cuda_device)
    compiled = torch.compile(lambda t: polar(t) * 2.0, fullgraph=True, backend="aot_eager")
    got = compiled(X)
    assert torch.equal(got, polar(X) * 2.0)


def test_run_with_operator_backend_under_torch_compile(cuda_device):
    table = coefficients.PS2_55
    buffers = polar_switch.validate_table(table, 1e-7)
    X = seeded((2, 128, 384), 96).to(cuda_device)
    compiled = torch.compile(lambda t: polar_switch._run(t, table, torch_ops.compiled_ops, 1e-7, buffers),
                             fullgraph=True, backend="aot_eager")
    assert torch.equal(compiled(X), polar_switch._run(X, table, cuda_ops, 1e-7, buffers))
