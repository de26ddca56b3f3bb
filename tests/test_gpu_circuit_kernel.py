"""The whole-circuit kernel (ps_set_circuit_kernel(1)): every stage of every
problem of a grouped call -- each matrix's Gram, inner iterations and apply,
for all outer iterations -- in one persistent CTA-pair launch, the stages of
a matrix chained through per-matrix completion counters with bounded waits.

Each tile is computed as the per-stage launches compute it, so results must
be the same bits as the per-stage path (ps_set_circuit_kernel(0)) for every
table shape (two and three buffers, residual applies of Polar Express, one
to five inner iterations), wide, tall and square inputs, padded shapes whose
final apply goes through the FP16 workspace, every output dtype, Muon updates
folded into the last apply, and a grouped call with more problems than one
launch takes (which falls back to per-stage launches). The per-stage path's
parity with the oracle is tested in test_gpu_circuit.py / test_gpu_large.py.
"""

import pytest
import torch

from polar_switch import _native as nat
from polar_switch import make_polynomial_orthogonalizer
from tests._util import seeded

pytestmark = pytest.mark.gpu


def _both(fn):
    """fn() with the whole-circuit kernel, then with per-stage launches."""
    prev = nat.set_circuit_kernel(1)
    try:
        on = fn()
        torch.cuda.synchronize()
        nat.set_circuit_kernel(0)
        off = fn()
        torch.cuda.synchronize()
    finally:
        nat.set_circuit_kernel(prev)
    return on, off


def _banks(shapes, seed, dtype=torch.float32, device="cuda"):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(*s, generator=g).to(dtype).to(device) for s in shapes]


CASES = [
    ("PS2_55", torch.float32, [(1, 2048, 1024), (2, 1024, 1024), (1, 1024, 2048), (2, 3072, 1024),
                               (1, 1024, 3072)]),
    ("PS3_55", torch.bfloat16, [(6, 768, 768), (2, 768, 3072), (2, 3072, 768)]),
    ("PS2_55", torch.float16, [(30, 256, 256), (3, 128, 640)]),
    ("POLAR_EXPRESS", torch.float32, [(3, 384, 512), (2, 512, 256)]),
    ("PS3_55", torch.float32, [(3, 130, 66), (2, 200, 136)]),   # padded: final apply via Xh
    ("PS2_64", torch.float32, [(1, 2048, 2048)]),
    ("PS2_11111", torch.float32, [(4, 256, 640)]),
]


@pytest.mark.parametrize("method,dtype,shapes", CASES,
                         ids=[f"{m}-{str(d)[6:]}-{len(s)}" for m, d, s in CASES])
def test_circuit_kernel_equals_per_stage_launches(cuda_device, method, dtype, shapes):
    banks = _banks(shapes, 21, dtype, cuda_device)
    polar = make_polynomial_orthogonalizer(method)
    on, off = _both(lambda: polar.grouped(banks))
    for a, b, s in zip(on, off, shapes):
        assert a.dtype == dtype and torch.equal(a, b), f"{method} {s}: circuit kernel differs"
    assert nat.get_status() == 0


def test_circuit_kernel_single_call_and_launch_count(cuda_device):
    X = seeded((4, 512, 1024), 22).to(cuda_device)
    polar = make_polynomial_orthogonalizer("PS2_55")
    on, off = _both(lambda: polar(X))
    assert torch.equal(on, off)
    prev = nat.set_circuit_kernel(1)
    try:
        n0 = nat.launch_count()
        nat.profile_enable(True)
        polar(X)
        prof = nat.profile_read()
        nat.profile_enable(False)
    finally:
        nat.set_circuit_kernel(prev)
    # two normalisation passes and one launch for the whole circuit
    assert nat.launch_count() - n0 == 3
    assert prof["circuit"]["launches"] == 1 and prof["square"]["launches"] == 0
    assert prof["circuit"]["flops"] == pytest.approx(4 * (22 * 512 ** 3))


def test_circuit_kernel_with_folded_muon_update(cuda_device):
    shapes = [(3, 256, 512), (2, 384, 128), (4, 192, 192)]
    dirs = _banks(shapes, 23, torch.bfloat16, cuda_device)
    polar = make_polynomial_orthogonalizer("PS2_55")
    base = _banks(shapes, 24, torch.float32, cuda_device)
    factors = [(0.998, -0.013), (0.999, -0.02), (1.0, -0.007)]

    def run():
        banks = [b.clone() for b in base]
        polar.grouped(dirs, updates=[(b, d, a) for b, (d, a) in zip(banks, factors)])
        return banks

    on, off = _both(run)
    for a, b in zip(on, off):
        assert torch.equal(a, b)


def test_more_problems_than_one_launch_fall_back(cuda_device):
    shapes = [(1, 128, 128 + 64 * i) for i in range(10)]  # 10 problems > 8 per launch
    banks = _banks(shapes, 25, torch.float32, cuda_device)
    polar = make_polynomial_orthogonalizer("PS2_55")
    on, off = _both(lambda: polar.grouped(banks))
    for a, b in zip(on, off):
        assert torch.equal(a, b)


def _packed_outputs(shapes, device, pad=128):
    """FP16 outputs packed into one buffer (each start 256-byte aligned), as a
    sharded step's receive segment holds them; returns (buffer, views)."""
    sizes = [L * r * c for L, r, c in shapes]
    offs, off = [], 0
    for n in sizes:
        offs.append(off)
        off += -(-n // pad) * pad
    buf = torch.full((off,), float("nan"), dtype=torch.float16, device=device)
    views = [buf[o:o + n].view(*s) for o, n, s in zip(offs, sizes, shapes)]
    return buf, views


PUSH_CASES = [
    ("PS2_55", [(4, 2048, 1024), (7, 1024, 1024), (4, 1024, 2048), (7, 3072, 1024), (4, 1024, 3072)],
     [1.0, 1.0, 1.0]),
    ("PS3_55", [(6, 768, 768), (2, 768, 3072), (2, 3072, 768)], [1.0, 2.0]),
    ("PS2_55", [(5, 256, 512), (3, 128, 128), (2, 136, 200)], [1.0]),
]


@pytest.mark.parametrize("method,shapes,phases", PUSH_CASES,
                         ids=[f"{m}-{len(s)}-{len(p)}" for m, s, p in PUSH_CASES])
def test_push_stores_results_into_peer_buffers(cuda_device, method, shapes, phases):
    """ps_circuit_grouped_push on one GPU, with other buffers of this GPU in
    place of the peers' copies: the local outputs equal ps_circuit_grouped's
    bit for bit (phased schedule included), and every 'peer' buffer holds the
    same bits at the same offsets (nothing outside the outputs written)."""
    from polar_switch.distributed import phase_ends
    banks = _banks(shapes, 26, torch.float32, cuda_device)
    polar = make_polynomial_orthogonalizer(method)
    want = [y.half() if y.dtype != torch.float16 else y
            for y in polar.grouped(banks, outs=[torch.empty(b.shape, dtype=torch.float16,
                                                            device=cuda_device) for b in banks])]
    local, outs = _packed_outputs(shapes, cuda_device)
    peers = [torch.full_like(local, float("nan")) for _ in range(3)]
    push = {"local": local.data_ptr(), "peers": [p.data_ptr() for p in peers],
            "phase_ends": phase_ends([s[0] for s in shapes], phases)}
    for _ in range(2):  # a second call over the same buffers
        polar.grouped(banks, outs=outs, push=push)
    torch.cuda.synchronize()
    assert nat.get_status() == 0
    for o, w, s in zip(outs, want, shapes):
        assert torch.equal(o, w), f"{method} {s}: pushed launch differs from ps_circuit_grouped"
    for p in peers:
        assert torch.equal(torch.isnan(p), torch.isnan(local))
        m = ~torch.isnan(local)
        assert torch.equal(p[m], local[m])


def test_push_refuses_what_one_launch_cannot_hold(cuda_device):
    polar = make_polynomial_orthogonalizer("PS2_55")
    # padded shape: the final apply would go through the workspace
    X = seeded((2, 130, 66), 27).to(cuda_device)
    local = torch.empty(2 * 130 * 66 + 128, dtype=torch.float16, device=cuda_device)
    out = local[:2 * 130 * 66].view(2, 130, 66)
    push = {"local": local.data_ptr(), "peers": [torch.empty_like(local).data_ptr()],
            "phase_ends": [[2]]}
    with pytest.raises(nat.NativeError) as e:
        polar.grouped([X], outs=[out], push=push)
    assert e.value.code == nat.PS_ERR_UNSUPPORTED
    # the whole-circuit kernel switched off
    prev = nat.set_circuit_kernel(0)
    try:
        Y = seeded((2, 128, 64), 28).to(cuda_device)
        with pytest.raises(nat.NativeError) as e:
            polar.grouped([Y], outs=[local[:2 * 128 * 64].view(2, 128, 64)], push=push)
        assert e.value.code == nat.PS_ERR_UNSUPPORTED
    finally:
        nat.set_circuit_kernel(prev)


def test_signal_flags_release_a_waiting_stream(cuda_device):
    """ps_circuit_grouped_signal: outputs equal ps_circuit_grouped's, every
    phase flag ends at 1 with its counter at the expected count, and a side
    stream that waits on each flag (ps_stream_wait_flag) and then copies that
    phase's outputs gets the final values."""
    from polar_switch.distributed import phase_ends
    shapes = [(6, 512, 256), (5, 256, 256), (4, 256, 768)]
    banks = _banks(shapes, 29, torch.float32, cuda_device)
    polar = make_polynomial_orthogonalizer("PS2_55")
    want = polar.grouped(banks, outs=[torch.empty(b.shape, dtype=torch.float16, device=cuda_device)
                                      for b in banks])
    phases = [1.0, 1.0, 2.0]
    ends = phase_ends([s[0] for s in shapes], phases)
    flags = torch.zeros(2 * len(phases) + 1, dtype=torch.int32, device=cuda_device)
    outs = [torch.full(b.shape, float("nan"), dtype=torch.float16, device=cuda_device) for b in banks]
    copies = [torch.full_like(o, float("nan")) for o in outs]
    side = torch.cuda.Stream(device=cuda_device)
    main = torch.cuda.current_stream(cuda_device)
    for _ in range(2):
        flags.zero_()
        side.wait_stream(main)
        polar.grouped(banks, outs=outs, signal={"flags": flags, "phase_ends": ends})
        with torch.cuda.stream(side):
            for k in range(len(phases)):
                nat.stream_wait_flag(side, flags.data_ptr() + 4 * k, 1)
                for o, c, e in zip(outs, copies, ends):
                    lo = e[k - 1] if k else 0
                    c[lo:e[k]].copy_(o[lo:e[k]], non_blocking=True)
        main.wait_stream(side)
        torch.cuda.synchronize()
        assert nat.get_status() == 0
        f = flags.cpu()
        assert f[:len(phases)].tolist() == [1] * len(phases)
        assert int(f[-1]) > 0  # every CTA counted itself out
        for o, c, w in zip(outs, copies, want):
            assert torch.equal(o, w) and torch.equal(c, w)
