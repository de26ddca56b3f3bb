"""GPU tests of Gram Newton-Schulz, the grouped (multi-shape) circuit used by
the Muon step, the sharded orthogonalizer at world size 1, and the device
status word of the bounded waits."""

import pytest
import torch

from oracle import circuit as oc
from oracle import gns as og
from polar_switch import coefficients
from tests._util import seeded

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(2, 128, 384), (256, 96), (3, 64, 200)])
def test_gns_rectangular(cuda_device, shape):
    from polar_switch import make_polynomial_orthogonalizer
    from polar_switch.gram_newton_schulz import GNS_COEFFICIENTS
    X = seeded(shape, 30)
    polar = make_polynomial_orthogonalizer("GNS")
    got = polar(X.to(cuda_device)).cpu()
    assert polar.last_execution["dispatch"] == "rectangular_gram"
    assert polar.last_execution["effective"] == "GNS"
    ref64 = og.gns_run(X, GNS_COEFFICIENTS, acc=torch.float64)
    ref32 = og.gns_run(X, GNS_COEFFICIENTS, acc=torch.float32)
    err = oc.relative_frobenius(got, ref64)
    floor = oc.relative_frobenius(ref32, ref64)
    assert err <= max(5e-3, 1.5 * floor), (err, floor)
    lo, hi = oc.singular_interval(got)
    rlo, rhi = oc.singular_interval(ref64)
    assert abs(lo - rlo) <= 1e-3 and abs(hi - rhi) <= 1e-3
    # published GNS interval [0.787021, 1.212979] for sigma in [1e-3, 1]
    assert 0.787 - 2e-3 <= lo and hi <= 1.213 + 2e-3


@pytest.mark.parametrize("shape", [(2, 256, 768), (3, 384, 128), (1, 1024, 2048), (2, 136, 200),
                                   (1, 2048, 512)])
def test_gns_one_call_matches_op_by_op(cuda_device, shape):
    """ps_gns runs the whole recurrence in one call; the result equals the
    op-by-op recurrence through the public kernels bit for bit."""
    from polar_switch.gram_newton_schulz import gram_newton_schulz, gram_newton_schulz_ops
    X = seeded(shape, 90).to(cuda_device)
    assert torch.equal(gram_newton_schulz(X), gram_newton_schulz_ops(X))


def test_gns_padded_shape_against_oracle(cuda_device):
    """Dimensions that are not multiples of 8 are zero-padded inside ps_gns."""
    from polar_switch import make_polynomial_orthogonalizer
    from polar_switch.gram_newton_schulz import GNS_COEFFICIENTS
    X = seeded((2, 130, 66), 91)
    got = make_polynomial_orthogonalizer("GNS")(X.to(cuda_device)).cpu()
    ref64 = og.gns_run(X, GNS_COEFFICIENTS, acc=torch.float64)
    ref32 = og.gns_run(X, GNS_COEFFICIENTS, acc=torch.float32)
    err = oc.relative_frobenius(got, ref64)
    floor = oc.relative_frobenius(ref32, ref64)
    assert err <= max(5e-3, 1.5 * floor), (err, floor)


def test_gns_square_uses_polar_express(cuda_device):
    from polar_switch import make_polynomial_orthogonalizer
    X = seeded((192, 192), 31)
    polar = make_polynomial_orthogonalizer("GNS")
    got = polar(X.to(cuda_device)).cpu()
    assert polar.last_execution["dispatch"] == "square_polar_express"
    assert polar.last_execution["effective"] == "POLAR_EXPRESS"
    ref = oc.run_circuit(X, coefficients.POLAR_EXPRESS, acc=torch.float64)
    assert oc.relative_frobenius(got, ref) <= 5e-3


def test_grouped_matches_single_calls(cuda_device):
    """Muon buckets of different shapes in one grouped call = separate calls, bit for bit."""
    from polar_switch import make_polynomial_orthogonalizer
    polar = make_polynomial_orthogonalizer("PS2_55")
    banks = [seeded((3, 256, 128), 40), seeded((2, 128, 128), 41), seeded((2, 128, 384), 42),
             seeded((1, 200, 96), 43), seeded((4, 64, 256), 44).to(torch.bfloat16)]
    banks = [b.to(cuda_device) for b in banks]
    grouped = polar.grouped(banks)
    for b, g in zip(banks, grouped):
        single = polar(b)
        assert g.dtype == b.dtype and g.shape == b.shape
        assert torch.equal(g, single)


def test_grouped_many_buckets_batched_launches(cuda_device):
    """More buckets than one launch takes (8 problems per launch): every
    bucket still equals its own call bit for bit. On the one-CTA kernel the
    Grams and applies of all buckets run in a few batched launches per outer
    iteration; on CTA pairs (the default) in one launch per bucket."""
    from polar_switch import _native as nat
    from polar_switch import make_polynomial_orthogonalizer
    polar = make_polynomial_orthogonalizer("PS2_55")
    shapes = [(2, 256, 128), (1, 128, 256), (2, 136, 136), (1, 384, 128), (3, 128, 128),
              (1, 128, 512), (2, 264, 128), (1, 128, 200), (2, 520, 128), (1, 128, 640)]
    banks = [seeded(s, 47 + i).to(cuda_device) for i, s in enumerate(shapes)]
    prev = nat.set_cta_pairs(0)
    try:
        nat.profile_enable(True)
        grouped = polar.grouped(banks)
        prof = nat.profile_read()
        nat.profile_enable(False)
        singles = [polar(b) for b in banks]
    finally:
        nat.set_cta_pairs(prev)
    # 2 outer iterations; per iteration Grams: tall and wide variants (5 problems each),
    # applies: one variant for all 10 problems -> 2 launches of 8 + 2
    assert prof["gram"]["launches"] == 2 * 2
    assert prof["apply"]["launches"] == 2 * 2
    nat.profile_enable(True)
    grouped_pairs = polar.grouped(banks)
    prof_pairs = nat.profile_read()
    nat.profile_enable(False)
    assert prof_pairs["gram"]["launches"] == 2 * len(shapes)
    assert prof_pairs["apply"]["launches"] == 2 * len(shapes)
    for b, g in zip(banks, grouped_pairs):
        assert torch.equal(g, polar(b))
    # the normalisations: 8 + 2 problems of one input type, two passes each
    assert prof["normalize"]["launches"] == 2 * 2
    for g, single in zip(grouped, singles):
        assert torch.equal(g, single)


def test_grouped_normalisations_batched_by_type(cuda_device):
    """The normalisations of a grouped call run as one launch per pass for all
    problems of one input type; strided, padded and mixed-type banks still
    equal their own calls bit for bit."""
    from polar_switch import _native as nat
    from polar_switch import make_polynomial_orthogonalizer
    polar = make_polynomial_orthogonalizer("PS3_55")
    banks = [seeded((2, 128, 256), 81).to(torch.bfloat16), seeded((1, 200, 96), 82).to(torch.bfloat16),
             seeded((192, 256), 80).t(), seeded((3, 128, 128), 83), seeded((1, 64, 72), 84).half(),
             seeded((2, 130, 66), 85)]
    banks = [b.to(cuda_device) for b in banks]
    assert not banks[2].is_contiguous()
    nat.profile_enable(True)
    grouped = polar.grouped(banks)
    prof = nat.profile_read()
    nat.profile_enable(False)
    # bf16 (2 problems), f32 (3) and f16 (1): two passes each
    assert prof["normalize"]["launches"] == 3 * 2
    for b, g in zip(banks, grouped):
        assert g.dtype == b.dtype and g.shape == b.shape
        assert torch.equal(g, polar(b))


def test_grouped_fp16_outputs(cuda_device):
    from polar_switch import make_polynomial_orthogonalizer
    polar = make_polynomial_orthogonalizer("PS3_55")
    banks = [seeded((2, 256, 128), 45).to(cuda_device), seeded((3, 128, 256), 46).to(cuda_device)]
    outs = [torch.empty(b.shape, device=cuda_device, dtype=torch.float16) for b in banks]
    polar.grouped(banks, outs=outs)
    for b, o in zip(banks, outs):
        assert torch.equal(o.float(), polar(b))


def test_sharded_world1_matches_polar(cuda_device):
    from polar_switch import make_polynomial_orthogonalizer
    from polar_switch.distributed import ShardedOrthogonalizer
    shapes = [(3, 256, 128), (4, 128, 128), (2, 128, 384)]
    banks = [seeded(s, 50 + i).to(cuda_device) for i, s in enumerate(shapes)]
    sharded = ShardedOrthogonalizer(shapes, method="PS2_55", device=cuda_device, world_size=1, rank=0)
    sharded(banks)
    polar = make_polynomial_orthogonalizer("PS2_55")
    for b, full in zip(banks, sharded.gathered_banks()):
        assert torch.equal(full.float(), polar(b))


def test_sharded_step_cuda_graph_replay(cuda_device):
    """A step captured as a CUDA graph and replayed on new contents of the same
    bank tensors gives the eager result bit for bit."""
    from polar_switch.distributed import ShardedOrthogonalizer
    shapes = [(3, 256, 128), (4, 128, 128), (2, 128, 384)]
    banks = [seeded(s, 60 + i).to(cuda_device) for i, s in enumerate(shapes)]
    step = ShardedOrthogonalizer(shapes, method="PS3_55", device=cuda_device, world_size=1, rank=0)
    step.capture(banks)
    for i, b in enumerate(banks):  # new inputs in the captured tensors
        b.copy_(seeded(b.shape, 70 + i).to(cuda_device))
    step.replay()
    torch.cuda.synchronize()
    graphed = [t.clone() for t in step.gathered_banks()]
    step(banks)
    eager = step.gathered_banks()
    for g, e in zip(graphed, eager):
        assert torch.equal(g, e)
    step.close()


def test_sharded_step_from_host_memory(cuda_device):
    """step_host: pinned host banks in, pinned FP16 results out, bucket by
    bucket with overlapped copies; equal to the device-resident step."""
    from polar_switch.distributed import ShardedOrthogonalizer
    shapes = [(3, 256, 128), (4, 128, 128), (2, 128, 384), (5, 264, 128)]
    host = [seeded(s, 80 + i).pin_memory() for i, s in enumerate(shapes)]
    step = ShardedOrthogonalizer(shapes, method="PS2_55", device=cuda_device, world_size=1, rank=0,
                                 buckets=3)
    out = step.step_host(host)
    torch.cuda.synchronize()
    got = out.clone()
    out2 = step.step_host(host, out)  # second call reuses the staging and the output buffer
    torch.cuda.synchronize()
    assert out2.data_ptr() == out.data_ptr() and torch.equal(out2, got)
    ref = ShardedOrthogonalizer(shapes, method="PS2_55", device=cuda_device, world_size=1, rank=0,
                                buckets=3)
    ref([h.to(cuda_device) for h in host])
    assert torch.equal(got, ref.recv.cpu())
    step.close()
    ref.close()


def test_status_word_and_bounded_wait(cuda_device):
    """A kernel whose wait can never complete gives up after its limit and
    records status 5; the context stays usable afterwards."""
    from polar_switch import _native as nat
    with torch.cuda.device(cuda_device):
        assert nat.get_status(clear=True) in (0, 5)
        assert nat.get_status() == 0
        nat.selftest_wait(2_000_000)  # ~1 ms of SM clock
        torch.cuda.synchronize()
        assert nat.get_status() == 5
        assert nat.get_status(clear=True) == 5
        assert nat.get_status() == 0
        # the device still computes correctly after the timed-out kernel
        from polar_switch import make_polynomial_orthogonalizer
        X = seeded((128, 256), 60)
        got = make_polynomial_orthogonalizer("PS2_55")(X.to(cuda_device)).cpu()
        ref = oc.run_circuit(X, coefficients.PS2_55, acc=torch.float64)
        assert oc.relative_frobenius(got, ref) <= 5e-3
        assert nat.get_status() == 0


def test_launch_counter_and_profiler(cuda_device):
    from polar_switch import _native as nat
    from polar_switch import make_polynomial_orthogonalizer
    polar = make_polynomial_orthogonalizer("PS2_55")
    X = seeded((2, 256, 512), 61).to(cuda_device)
    prev_circ = nat.set_circuit_kernel(0)  # per-stage launches, counted below
    for chain, squares in ((0, 10), (1, 2)):
        prev = nat.set_chain(chain)
        try:
            n0 = nat.launch_count()
            nat.profile_enable(True)
            polar(X)
            prof = nat.profile_read()
            nat.profile_enable(False)
        finally:
            nat.set_chain(prev)
        # 2 normalise + 2 x (1 gram + 5 squares (or one chain launch) + 1 apply)
        assert nat.launch_count() - n0 == 6 + squares
        assert prof["normalize"]["launches"] == 2
        assert prof["gram"]["launches"] == 2 and prof["square"]["launches"] == squares
        assert prof["apply"]["launches"] == 2
        assert prof["square"]["flops"] == pytest.approx(10 * 2 * 256 ** 3)
        assert all(v["ms"] > 0 for v in prof.values() if v["launches"])
    nat.set_circuit_kernel(prev_circ)
