"""The chain kernel: all inner iterations of an outer iteration in one
persistent launch on CTA pairs, a matrix's next step starting once its
previous step is stored (per-matrix completion counters, bounded waits).

Each tile is computed as the per-iteration CTA-pair launches compute it, so
the whole circuit must give the same bits with the chain on and off
(ps_set_chain(1) / ps_set_chain(0)), for every table shape the circuits use:
two and three buffers, one to five inner iterations, more inner iterations
than one chain launch takes, ragged and small n, single matrices, batches
across several n-groups, and larger n on CTA pairs (ps_set_cta_pairs(1)).
The parity of the per-iteration path with the oracle is tested elsewhere
(test_gpu_circuit.py, test_gpu_large.py); test_chain_against_oracle checks one
case directly. A wait on a counter that never arrives runs out and reports
status 6 (ps_selftest_chain_wait), leaving the device usable.
"""

import pytest
import torch

from oracle import circuit as oc
from polar_switch import _native as nat
from polar_switch import coefficients, make_polynomial_orthogonalizer
from tests._util import seeded

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def per_stage_launches():
    """The chain is the inner-iteration launch of the per-stage path; the
    whole-circuit kernel (the default) replaces it, so these tests run with
    per-stage launches."""
    prev = nat.set_circuit_kernel(0)
    yield
    nat.set_circuit_kernel(prev)


def _both(fn):
    """fn() with the chain on, then off; restores the previous mode."""
    prev = nat.set_chain(1)
    try:
        on = fn()
        torch.cuda.synchronize()
        nat.set_chain(0)
        off = fn()
        torch.cuda.synchronize()
    finally:
        nat.set_chain(prev)
    return on, off


def _banks(shapes, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(*s, generator=g) * scale for s in shapes]


CASES = [
    ("PS2_55", [(1, 2048, 1024), (2, 1024, 1024), (1, 1024, 2048), (2, 3072, 1024), (1, 1024, 3072)]),
    ("PS3_55", [(8, 768, 768), (2, 768, 3072), (2, 3072, 768)]),
    ("PS2_55", [(40, 256, 256)]),
    ("PS3_55", [(3, 130, 66), (5, 200, 136)]),
    ("PS2_55", [(1, 512, 1024)]),
    ("POLAR_EXPRESS", [(3, 384, 512)]),
    ("PS2_11111", [(4, 256, 640)]),
    ("PS3_64", [(6, 512, 512), (2, 256, 1024)]),
]


@pytest.mark.parametrize("method,shapes", CASES, ids=[f"{m}-{len(s)}banks-{s[0][1]}" for m, s in CASES])
def test_chain_equals_per_iteration_launches(cuda_device, method, shapes):
    banks = [b.to(cuda_device) for b in _banks(shapes, 11)]
    polar = make_polynomial_orthogonalizer(method)
    on, off = _both(lambda: polar.grouped(banks))
    for a, b, s in zip(on, off, shapes):
        assert torch.equal(a, b), f"{method} {s}: chain and per-iteration launches differ"
    assert nat.get_status() == 0


def test_chain_single_call_and_more_steps_than_one_launch(cuda_device):
    """polar(X) goes through the same path; a table with 10 inner iterations
    takes two chain launches (8 + 2) in one outer iteration."""
    X = seeded((6, 384, 768), 12).to(cuda_device)
    polar = make_polynomial_orthogonalizer("PS2_55")
    on, off = _both(lambda: polar(X))
    assert torch.equal(on, off)
    steps = tuple((1 - k % 2, k % 2, 1 - k % 2, 0.5, 0.5, 0.01 * k) for k in range(10))
    table = ((0.0, ((1, 0, 0, 1.0, 0.25, 0.0),) + steps[1:]),)
    custom = make_polynomial_orthogonalizer(table)
    on, off = _both(lambda: custom(X))
    assert torch.equal(on, off)
    assert nat.get_status() == 0


@pytest.mark.parametrize("method,shape", [("PS3_55", (2, 1152, 2304)), ("PS2_55", (1, 2048, 2048)),
                                          ("PS2_55", (3, 1024, 1536)), ("PS3_55", (2, 1088, 1088))])
def test_chain_on_pairs_for_larger_n(cuda_device, method, shape):
    """With every product on CTA pairs (ps_set_cta_pairs(1)) the chain also
    takes n > 1024 (more pair tiles per matrix, a ragged last pair block)."""
    X = seeded(shape, 13).to(cuda_device)
    polar = make_polynomial_orthogonalizer(method)
    prev = nat.set_cta_pairs(1)
    try:
        on, off = _both(lambda: polar(X))
    finally:
        nat.set_cta_pairs(prev)
    assert torch.equal(on, off)
    assert nat.get_status() == 0


def test_chain_against_oracle(cuda_device):
    X = seeded((4, 1024, 1024), 14)
    polar = make_polynomial_orthogonalizer("PS3_55")
    prev = nat.set_chain(1)
    try:
        got = polar(X.to(cuda_device)).cpu()
    finally:
        nat.set_chain(prev)
    table = coefficients.PS3_55
    for i in (0, 3):
        ref64 = oc.run_circuit(X[i], table, acc=torch.float64)
        ref32 = oc.run_circuit(X[i], table, acc=torch.float32)
        err = oc.relative_frobenius(got[i], ref64)
        floor = oc.relative_frobenius(ref32, ref64)
        assert err <= max(5e-3, 1.5 * floor), (err, floor)


def test_chain_dependency_wait_runs_out_and_reports(cuda_device):
    """A chain whose second step waits for a count that never arrives: the
    waits give up after ~1 ms of SM clock, status 6 is recorded, and the
    device keeps computing correctly afterwards."""
    lib = nat.load()
    ws = torch.empty(1 << 20, dtype=torch.uint8, device=cuda_device)
    with torch.cuda.device(cuda_device):
        nat.get_status(clear=True)
        rc = lib.ps_selftest_chain_wait(nat.ptr(ws), ws.numel(), 2_000_000, nat.stream_ptr(cuda_device))
        assert rc == nat.PS_OK, lib.ps_last_error()
        torch.cuda.synchronize()
        assert nat.get_status() == 6
        assert nat.get_status(clear=True) == 6
        assert nat.get_status() == 0
        X = seeded((2, 256, 512), 15)
        got = make_polynomial_orthogonalizer("PS2_55")(X.to(cuda_device)).cpu()
        ref = oc.run_circuit(X, coefficients.PS2_55, acc=torch.float64)
        assert oc.relative_frobenius(got, ref) <= 5e-3
        assert nat.get_status() == 0
