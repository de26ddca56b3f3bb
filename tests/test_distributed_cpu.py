"""Sharding plan and the gather logic of the multi-GPU Muon step, on CPU
ranks with the gloo backend (world size 2 and 4). The circuit itself is
replaced by the CPU oracle, so these tests exercise only the host-side logic:
plan, packing, in-place all-gather, unpacking, and failure handling."""

import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

from polar_switch import circuit_flops, coefficients
from polar_switch.distributed import (ShardedOrthogonalizer, gemma3_1b_banks, nanogpt_banks, plan_loads,
                                      plan_shards, qwen3_0_6b_banks)


def flops(r, c):
    return circuit_flops(coefficients.PS2_55, r, c)


@pytest.mark.parametrize("banks", [qwen3_0_6b_banks(), gemma3_1b_banks(), nanogpt_banks(),
                                   [(4, 8192, 28672)], [(3, 64, 64), (1, 128, 32)]])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_covers_every_matrix_once_and_balances(banks, world):
    slices = plan_shards(banks, world, flops)
    for g, (L, _, _) in enumerate(banks):
        covered = []
        for r in range(world):
            start, count = slices[r][g]
            covered.extend(range(start, start + count))
        assert covered == list(range(L))
    loads = plan_loads(banks, slices, flops)
    biggest = max(flops(r, c) for _, r, c in banks)
    # LPT: no rank exceeds the average load by more than one largest matrix
    assert max(loads) <= sum(loads) / world + biggest + 1e-6


def test_plan_is_deterministic():
    a = plan_shards(qwen3_0_6b_banks(), 8, flops)
    b = plan_shards(list(qwen3_0_6b_banks()), 8, flops)
    assert a == b


def test_qwen_plan_balance_at_8_ranks():
    banks = qwen3_0_6b_banks()
    loads = plan_loads(banks, plan_shards(banks, 8, flops), flops)
    assert max(loads) / (sum(loads) / 8) < 1.03


def _oracle_grouped(inputs, outs):
    from oracle import circuit as oc
    for X, Y in zip(inputs, outs):
        Y.copy_(oc.run_circuit(X, coefficients.PS2_55, out_dtype=torch.float16))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, shapes, result_queue, fail_rank):
    try:
        import datetime
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
        g = torch.Generator().manual_seed(7)
        banks = [torch.randn(*s, generator=g) for s in shapes]  # same on every rank
        step = ShardedOrthogonalizer(shapes, method="PS2_55", device="cpu", world_size=world, rank=rank,
                                     grouped_fn=_oracle_grouped)
        if rank == fail_rank:
            raise RuntimeError("injected failure on the host before the collective")
        step(banks)
        full = step.gathered_banks()
        result_queue.put((rank, [f.clone() for f in full]))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report to the parent instead of hanging it
        result_queue.put((rank, f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))


def _run(world, shapes, fail_rank=-1, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shapes, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, res = q.get(timeout=timeout)
            results[rank] = res
    finally:
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()
    return results


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_step_gloo_matches_single_process(world):
    shapes = [(5, 48, 32), (3, 32, 32), (2, 32, 80)]
    results = _run(world, shapes)
    assert sorted(results) == list(range(world))
    g = torch.Generator().manual_seed(7)
    banks = [torch.randn(*s, generator=g) for s in shapes]
    from oracle import circuit as oc
    expected = [oc.run_circuit(b, coefficients.PS2_55, out_dtype=torch.float16) for b in banks]
    for r in range(world):
        assert not isinstance(results[r], str), results[r]
        for got, exp in zip(results[r], expected):
            assert torch.equal(got, exp)


def test_rank_failure_before_collective_is_reported():
    """A rank that raises before the all-gather: the others end with an error
    from the process-group timeout instead of hanging."""
    shapes = [(4, 32, 32)]
    results = _run(2, shapes, fail_rank=1, timeout=180)
    assert isinstance(results[1], str) and "injected failure" in results[1]
    assert isinstance(results[0], str)  # the surviving rank saw the collective fail
