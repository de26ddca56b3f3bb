"""ShardedMuon's host logic on CPU ranks (gloo): the gradient scatter, the
momentum kept for the local chunk only, the grouped orthogonalization of the
local chunks and the gather of the updated slices, against one process that
applies the same update rule to the averaged gradients of whole banks.

The per-element math is the reference's (training/muon.py:64-86) written in
torch here, and the orthogonalization is the CPU oracle: the CUDA kernels are
exercised by the GPU tests. Gradients are multiples of 1/16 so their average
is exact in any summation order, which makes the comparison bit-exact."""

import datetime
import math
import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

from polar_switch import coefficients
from polar_switch.muon import ShardedMuon, check_banks, padded_count

MOMENTUM, LR, DECAY = 0.9, 0.02, 0.1


def _orthogonalize(X):
    from oracle import circuit as oc
    return oc.run_circuit(X, coefficients.PS2_55, out_dtype=torch.float16)


def _directions(grad, mom, momentum, out_dtype):
    mom.mul_(momentum).add_(grad)
    return grad.add(mom, alpha=momentum).to(out_dtype)


def _update(param, update, decay, alpha):
    param.mul_(decay)
    param.add_(update.to(param.dtype), alpha=alpha)


class _CpuShardedMuon(ShardedMuon):
    """ShardedMuon with the per-element steps in torch on CPU tensors."""

    def _directions(self, grad_chunk, mom_chunk, momentum, out_dtype):
        return _directions(grad_chunk, mom_chunk, momentum, out_dtype)

    def _update(self, param_chunk, update, decay, alpha):
        _update(param_chunk, update, decay, alpha)


class _RecordingLog:
    """Stands in for NormLog: keeps (label, shape, matrix_start) per record."""

    def __init__(self):
        self.calls = []

    def record(self, label, output, matrix_start=0, execution=None, matrix_names=None):
        self.calls.append((label, tuple(output.shape), matrix_start))


def _banks(shapes, padding):
    g = torch.Generator().manual_seed(11)
    banks = []
    for (count, r, c), pad in zip(shapes, padding):
        b = torch.randn(count, r, c, generator=g) * 0.1
        b[count - pad:] = 0
        banks.append(b)
    return banks


def _grads(shapes, padding, rank, step):
    g = torch.Generator().manual_seed(1000 * step + rank)
    out = []
    for (count, r, c), pad in zip(shapes, padding):
        x = torch.randint(-64, 65, (count, r, c), generator=g).float() / 16
        x[count - pad:] = 0  # padding matrices get no gradient
        out.append(x)
    return out


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, shapes, padding, steps, scale, q, fail_rank=-1):
    try:
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
        banks = [torch.nn.Parameter(b) for b in _banks(shapes, padding)]
        log = _RecordingLog()
        opt = _CpuShardedMuon(banks, _orthogonalize, lr=LR, momentum=MOMENTUM, weight_decay=DECAY,
                              scale=scale, norm_log=log)
        assert (opt.world_size, opt.rank) == (world, rank)
        if rank == fail_rank:
            raise RuntimeError("injected failure on the host before the step")
        for step in range(steps):
            for b, gr in zip(banks, _grads(shapes, padding, rank, step)):
                b.grad = gr
            opt.step()
        # numpy, not tensors: a tensor would travel as a shared-memory handle
        # that dies with this process
        moms = [opt.state[b]["momentum_chunk"].numpy().copy() for b in banks]
        n = [s[0] // world for s in shapes]
        assert log.calls == [(f"bank{i}", (n[i], *shapes[i][1:]), rank * n[i])
                             for _ in range(steps) for i in range(len(shapes))], log.calls
        q.put((rank, ([b.detach().numpy().copy() for b in banks], moms)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))


def _expected(shapes, padding, world, steps, scale):
    """One process, whole banks, gradients averaged over the ranks."""
    banks = _banks(shapes, padding)
    moms = [torch.zeros_like(b) for b in banks]
    for step in range(steps):
        per_rank = [_grads(shapes, padding, r, step) for r in range(world)]
        for i, bank in enumerate(banks):
            grad = torch.stack([per_rank[r][i] for r in range(world)]).sum(0) / world
            d = _directions(grad, moms[i], MOMENTUM, torch.bfloat16 if scale == "rms" else bank.dtype)
            u = _orthogonalize(d)
            rows, cols = bank.shape[-2:]
            factor = 0.2 * math.sqrt(max(rows, cols)) if scale == "rms" else math.sqrt(rows / cols)
            _update(bank, u, 1 - LR * DECAY, -LR * factor)
    return banks, moms


@pytest.mark.parametrize("world,shapes,padding,scale", [
    (2, [(4, 32, 48), (2, 64, 32), (6, 32, 32)], [0, 1, 1], "rms"),
    (4, [(4, 48, 32), (8, 32, 32)], [1, 3], "shape"),
])
def test_sharded_muon_gloo_matches_single_process(world, shapes, padding, scale):
    steps = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shapes, padding, steps, scale, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, res = q.get(timeout=180)
            results[rank] = res
    finally:
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()
    assert sorted(results) == list(range(world))
    exp_banks, exp_moms = _expected(shapes, padding, world, steps, scale)
    for r in range(world):
        assert not isinstance(results[r], str), results[r]
        banks, moms = ([torch.from_numpy(a) for a in part] for part in results[r])
        for got, exp, (count, _, _), pad in zip(banks, exp_banks, shapes, padding):
            assert torch.equal(got, exp)  # every rank holds every matrix after the gather
            assert not got[count - pad:].any()  # padding stays zero
        for got, exp, (count, _, _) in zip(moms, exp_moms, shapes):
            n = count // world
            assert torch.equal(got, exp[r * n:(r + 1) * n])  # momentum of the local chunk only


def test_rank_failure_before_the_step_is_reported():
    """A rank that raises before the step: the other ends with an error from
    its gradient scatter (peer gone, or the process-group timeout) instead of
    hanging."""
    shapes, padding = [(2, 32, 32)], [0]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, shapes, padding, 1, "rms", q, 1)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):
            rank, res = q.get(timeout=180)
            results[rank] = res
    finally:
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()
    assert isinstance(results[1], str) and "injected failure" in results[1]
    assert isinstance(results[0], str)  # the surviving rank's collective failed


def test_sharded_muon_world1_without_process_group():
    shapes, padding = [(3, 32, 48), (2, 32, 32)], [0, 0]
    banks = [torch.nn.Parameter(b) for b in _banks(shapes, padding)]
    opt = _CpuShardedMuon(banks, _orthogonalize, lr=LR, momentum=MOMENTUM, weight_decay=DECAY)
    assert (opt.world_size, opt.rank) == (1, 0)
    for b, gr in zip(banks, _grads(shapes, padding, 0, 0)):
        b.grad = gr
    opt.step()
    exp_banks, _ = _expected(shapes, padding, 1, 1, "rms")
    for got, exp in zip(banks, exp_banks):
        assert torch.equal(got.detach(), exp)


def test_sharded_muon_rejects_banks_that_do_not_split():
    check_banks([torch.zeros(4, 8, 8), torch.zeros(2, 8, 16)], 2)
    with pytest.raises(ValueError):
        check_banks([torch.zeros(3, 8, 8)], 2)
    with pytest.raises(ValueError):
        check_banks([torch.zeros(8, 8)], 1)
    with pytest.raises(ValueError):
        check_banks([torch.zeros(2, 8, 8).transpose(1, 2)], 1)
    with pytest.raises(ValueError):
        ShardedMuon([torch.nn.Parameter(torch.zeros(8, 8))], _orthogonalize, lr=LR)
    assert padded_count(20, 8) == 24 and padded_count(24, 8) == 24 and padded_count(1, 4) == 4


def test_sharded_muon_has_no_cpu_fallback():
    """Without the per-element overrides the step runs the CUDA kernels and
    refuses CPU banks."""
    bank = torch.nn.Parameter(torch.randn(2, 16, 16))
    bank.grad = torch.randn(2, 16, 16)
    opt = ShardedMuon([bank], _orthogonalize, lr=LR)
    with pytest.raises(NotImplementedError):
        opt.step()
