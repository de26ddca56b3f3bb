"""The B200 Muon optimizer: the fused momentum / Nesterov / stack / cast
kernel against torch's elementwise sequence, and whole optimizer steps against
the reference's update rule (training/muon.py:58-86, restated here)."""

import math

import pytest
import torch

from polar_switch import make_polynomial_orthogonalizer
from polar_switch.muon import Muon, muon_directions
from tests._util import fp16_ulp, seeded

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,out_dtype", [(torch.float32, torch.bfloat16), (torch.float32, torch.float32),
                                             (torch.bfloat16, torch.bfloat16)])
def test_fused_directions_match_torch(cuda_device, dtype, out_dtype):
    mu = 0.95
    grads = [seeded((192, 320), 400 + i, dtype=dtype).to(cuda_device) for i in range(5)]
    moms = [seeded((192, 320), 410 + i, dtype=dtype).to(cuda_device) for i in range(5)]
    ref_moms = [m.clone() for m in moms]
    ref_dirs = []
    for g, m in zip(grads, ref_moms):
        m.mul_(mu).add_(g)
        ref_dirs.append(g.add(m, alpha=mu))
    ref = torch.stack(ref_dirs).to(out_dtype)
    got = muon_directions(grads, moms, mu, out_dtype)
    for m, r in zip(moms, ref_moms):
        assert torch.equal(m, r)  # the momentum is rounded exactly where torch rounds it
    assert got.shape == ref.shape and got.dtype == out_dtype
    # g + mu * m may or may not be contracted into one FMA by torch: one rounding step apart at most
    g32, r32 = got.float(), ref.float()
    step = (fp16_ulp(r32) / 8) if out_dtype == torch.float32 else torch.pow(
        2.0, torch.floor(torch.log2(r32.abs().clamp_min(2.0 ** -126))) - 7)
    assert ((g32 - r32).abs() <= step + 1e-30).all()
    assert float((g32 != r32).float().mean()) < 0.01


@pytest.mark.parametrize("dtype,udtype", [(torch.float32, torch.bfloat16), (torch.bfloat16, torch.bfloat16),
                                          (torch.float32, torch.float16)])
def test_fused_update_matches_torch(cuda_device, dtype, udtype):
    from polar_switch.muon import muon_update
    params = [seeded((160, 264), 450 + i, dtype=dtype).to(cuda_device) for i in range(4)]
    update = torch.stack([seeded((160, 264), 460 + i).to(cuda_device) for i in range(4)]).to(udtype)
    ref = [p.clone() for p in params]
    decay, alpha = 1 - 0.02 * 0.1, -0.02 * 3.7
    for p, u in zip(ref, update.unbind()):
        p.mul_(decay)
        p.add_(u.to(p.dtype), alpha=alpha)
    muon_update(params, update, decay, alpha)
    for got, want in zip(params, ref):
        g, w = got.float(), want.float()
        # one rounding step of the parameter dtype at most (FMA or not in torch's add)
        step = torch.pow(2.0, torch.floor(torch.log2(w.abs().clamp_min(2.0 ** -126)))
                         - (23 if dtype == torch.float32 else 7))
        assert ((g - w).abs() <= step).all()
        assert float((g != w).float().mean()) < 0.01


def _reference_step(params, grads, moms, polar, lr, mu, wd):
    """training/muon.py:63-86 for one bucket of the "rms" scale."""
    directions = []
    for g, m in zip(grads, moms):
        m.mul_(mu).add_(g)
        directions.append(g.add(m, alpha=mu))
    update = polar(torch.stack(directions).bfloat16()).clone()
    rows, cols = params[0].shape
    factor = 0.2 * math.sqrt(max(rows, cols))
    for p, u in zip(params, update.unbind()):
        p.mul_(1 - lr * wd)
        p.add_(u.to(p.dtype), alpha=-lr * factor)


def test_optimizer_steps_follow_the_reference_rule(cuda_device):
    polar = make_polynomial_orthogonalizer("PS2_55")
    shapes = [(256, 512)] * 3 + [(384, 128)] * 2
    params = [torch.nn.Parameter(seeded(s, 420 + i).to(cuda_device) * 0.02) for i, s in enumerate(shapes)]
    ref_params = [p.detach().clone() for p in params]
    ref_moms = [torch.zeros_like(p) for p in ref_params]
    opt = Muon([{"params": params, "role": "mlp"}], polar, lr=0.02, weight_decay=0.1)
    for step in range(2):
        grads = [seeded(s, 440 + 10 * step + i).to(cuda_device) for i, s in enumerate(shapes)]
        for p, g in zip(params, grads):
            p.grad = g.clone()
        opt.step()
        for lo, hi in ((0, 3), (3, 5)):
            _reference_step(ref_params[lo:hi], grads[lo:hi], ref_moms[lo:hi], polar, 0.02, 0.95, 0.1)
    for p, r in zip(params, ref_params):
        assert float((p.detach() - r).norm() / r.norm()) < 1e-3


def test_sharded_muon_world1_equals_muon(cuda_device):
    """ShardedMuon on banks at world size 1 runs the same kernels on the same
    matrices as Muon on the banks' matrices as separate parameters: the same
    bits after two steps, padding matrices included (they stay zero)."""
    from polar_switch.muon import ShardedMuon
    shapes = [(3, 256, 128), (4, 128, 384), (2, 192, 192)]
    banks = [seeded(s, 500 + i).to(cuda_device) * 0.05 for i, s in enumerate(shapes)]
    banks[1][3:] = 0  # one padding matrix
    sharded = [torch.nn.Parameter(b.clone()) for b in banks]
    single = [torch.nn.Parameter(m.clone()) for b in banks for m in b.unbind(0)]
    polar = make_polynomial_orthogonalizer("PS2_55")
    opt_s = ShardedMuon(sharded, polar, lr=0.02, momentum=0.95, weight_decay=0.1)
    opt_m = Muon([{"params": single, "role": "all"}], polar, lr=0.02, momentum=0.95, weight_decay=0.1)
    assert opt_s.world_size == 1
    for step in range(2):
        grads = [seeded(s, 600 + 10 * step + i).to(cuda_device) for i, s in enumerate(shapes)]
        grads[1][3:] = 0
        for p, g in zip(sharded, grads):
            p.grad = g.clone()
        for p, g in zip(single, [m for g in grads for m in g.unbind(0)]):
            p.grad = g.clone()
        opt_s.step()
        opt_m.step()
    flat = [m for b in sharded for m in b.detach().unbind(0)]
    for a, b in zip(flat, single):
        assert torch.equal(a, b.detach())
    assert not sharded[1][3:].any()


def test_transposed_view_parameters_take_the_reference_sequence(cuda_device):
    """A parameter that is a transposed view has a momentum buffer with its
    strides (zeros_like keeps them); the reference accepts it, and so must the
    drop-in: same bits as the reference rule on the same orthogonalizer."""
    polar = make_polynomial_orthogonalizer("PS2_55")
    base = [seeded((384, 256), 700 + i).to(cuda_device) * 0.02 for i in range(3)]
    params = [torch.nn.Parameter(b.clone().mT) for b in base]  # (256, 384), not contiguous
    assert not params[0].is_contiguous()
    ref_params = [b.clone().mT for b in base]
    ref_moms = [torch.zeros_like(p) for p in ref_params]
    opt = Muon([{"params": params, "role": "attn"}], polar, lr=0.02, weight_decay=0.1)
    for step in range(2):
        grads = [seeded((256, 384), 710 + 10 * step + i).to(cuda_device) for i in range(3)]
        for p, g in zip(params, grads):
            p.grad = g.clone()
        opt.step()
        _reference_step(ref_params, grads, ref_moms, polar, 0.02, 0.95, 0.1)
    for p, r, m in zip(params, ref_params, ref_moms):
        assert torch.equal(p.detach(), r)
        assert torch.equal(opt.state[p]["momentum_buffer"], m)


def test_fp32_gradients_on_bf16_weights(cuda_device):
    """FP32 gradients on BF16 weights: the reference adds them into the BF16
    momentum buffer and forms FP32 directions; the drop-in keeps going the same
    way (momentum bit for bit, parameters within the fused update's rounding)."""
    polar = make_polynomial_orthogonalizer("PS2_55")
    shapes = [(256, 512)] * 2
    params = [torch.nn.Parameter((seeded(s, 720 + i) * 0.02).to(cuda_device, torch.bfloat16))
              for i, s in enumerate(shapes)]
    ref_params = [p.detach().clone() for p in params]
    ref_moms = [torch.zeros_like(p) for p in ref_params]
    opt = Muon([{"params": params, "role": "mlp"}], polar, lr=0.02, weight_decay=0.1)
    for step in range(2):
        grads = [seeded(s, 730 + 10 * step + i).to(cuda_device) for i, s in enumerate(shapes)]
        for p, g in zip(params, grads):
            p.grad_dtype = None  # torch checks a gradient's dtype unless told not to
            p.grad = g.clone()  # FP32 gradient on a BF16 parameter
        opt.step()
        _reference_step(ref_params, grads, ref_moms, polar, 0.02, 0.95, 0.1)
    for p, r, m in zip(params, ref_params, ref_moms):
        assert torch.equal(opt.state[p]["momentum_buffer"], m)
        assert float((p.detach().float() - r.float()).norm() / r.float().norm()) < 1e-3


@pytest.mark.parametrize("pdtype", [torch.float32, torch.bfloat16])
def test_update_folded_into_the_last_apply_equals_the_update_kernel(cuda_device, pdtype):
    """grouped(..., updates=...) applies p <- p * decay + alpha * u inside the
    circuit's last apply; it must give the bits of the circuit's output followed
    by ps_muon_update (itself tested against torch's sequence above)."""
    from polar_switch.muon import muon_update
    polar = make_polynomial_orthogonalizer("PS2_55")
    shapes = [(3, 256, 512), (2, 384, 128), (4, 192, 192)]
    dirs = [seeded(s, 800 + i).to(cuda_device).bfloat16() for i, s in enumerate(shapes)]
    banks = [(seeded(s, 810 + i) * 0.02).to(cuda_device, pdtype) for i, s in enumerate(shapes)]
    ref = [b.clone() for b in banks]
    factors = [(1 - 0.02 * 0.1, -0.02 * (0.2 * max(s[1:]) ** 0.5)) for s in shapes]
    outs = polar.grouped(dirs)
    for r, u, (decay, alpha) in zip(ref, outs, factors):
        muon_update(list(r.unbind(0)), u.contiguous(), decay, alpha)
    got = polar.grouped(dirs, updates=[(b, d, a) for b, (d, a) in zip(banks, factors)])
    assert all(o is None for o in got)
    for b, r in zip(banks, ref):
        assert torch.equal(b, r)


def test_sharded_muon_fused_update_equals_unfused(cuda_device):
    from polar_switch.muon import ShardedMuon
    shapes = [(3, 256, 128), (4, 128, 384), (2, 192, 192)]
    base = [seeded(s, 820 + i).to(cuda_device) * 0.05 for i, s in enumerate(shapes)]
    polar = make_polynomial_orthogonalizer("PS2_55")
    fused = [torch.nn.Parameter(b.clone()) for b in base]
    plain = [torch.nn.Parameter(b.clone()) for b in base]
    opt_f = ShardedMuon(fused, polar, lr=0.02, weight_decay=0.1, fuse_update=True)
    opt_p = ShardedMuon(plain, polar, lr=0.02, weight_decay=0.1, fuse_update=False)
    for step in range(2):
        grads = [seeded(s, 830 + 10 * step + i).to(cuda_device) for i, s in enumerate(shapes)]
        for p, q, gr in zip(fused, plain, grads):
            p.grad = gr.clone()
            q.grad = gr.clone()
        opt_f.step()
        opt_p.step()
    for a, b in zip(fused, plain):
        assert torch.equal(a.detach(), b.detach())
