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


def _worker(rank, world, port, shapes, result_queue, fail_rank, buckets=None):
    try:
        import datetime
        import torch.distributed as dist
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
        g = torch.Generator().manual_seed(7)
        banks = [torch.randn(*s, generator=g) for s in shapes]  # same on every rank
        step = ShardedOrthogonalizer(shapes, method="PS2_55", device="cpu", world_size=world, rank=rank,
                                     grouped_fn=_oracle_grouped, buckets=buckets)
        if rank == fail_rank:
            raise RuntimeError("injected failure on the host before the collective")
        step(banks)
        full = step.gathered_banks()
        result_queue.put((rank, [f.clone() for f in full]))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report to the parent instead of hanging it
        result_queue.put((rank, f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))


def _run(world, shapes, fail_rank=-1, timeout=120, buckets=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shapes, q, fail_rank, buckets)) for r in range(world)]
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


@pytest.mark.parametrize("world,buckets", [(2, None), (4, None), (2, 1), (3, 3)])
def test_sharded_step_gloo_matches_single_process(world, buckets):
    shapes = [(5, 48, 32), (3, 32, 32), (2, 32, 80)]
    results = _run(world, shapes, buckets=buckets)
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


@pytest.mark.parametrize("banks", [qwen3_0_6b_banks(), gemma3_1b_banks(), nanogpt_banks(), [(4, 8192, 28672)],
                                   [(3, 64, 64), (1, 128, 32)], [(1, 256, 256)]])
@pytest.mark.parametrize("buckets", [1, 2, 4, 7, [1, 3, 3, 1]])
def test_buckets_cover_every_matrix_once(banks, buckets):
    from polar_switch.distributed import plan_buckets
    plan = plan_buckets(banks, buckets, flops)
    nb = buckets if isinstance(buckets, int) else len(buckets)
    assert 1 <= len(plan) <= nb
    seen = [[] for _ in banks]
    for pieces in plan:
        assert pieces
        for g, start, count in pieces:
            assert count > 0
            seen[g].extend(range(start, start + count))
    assert seen == [list(range(L)) for L, _, _ in banks]
    if isinstance(buckets, int) and sum(L for L, _, _ in banks) >= 8 * buckets:
        costs = [sum(c * flops(*banks[g][1:]) for g, _, c in p) for p in plan]
        biggest = max(flops(r, c) for _, r, c in banks)
        assert max(costs) <= sum(costs) / buckets + biggest + 1e-6


@pytest.mark.parametrize("buckets", [1, 3])
def test_bucketed_layout_single_rank_views(buckets):
    """Offsets of the bucketed receive buffer: every rank's views are disjoint,
    16-byte aligned, and together cover each bank once."""
    shapes = qwen3_0_6b_banks()
    world = 4
    views = []
    for r in range(world):
        step = ShardedOrthogonalizer(shapes, method="PS2_55", device="meta", world_size=world, rank=r,
                                     grouped_fn=_oracle_grouped, buckets=buckets)
        for plan in step.plans:
            for g, start, v in step._segment_views(plan, r):
                off = v.storage_offset()
                assert off % 8 == 0
                views.append((off, off + v.numel(), g, start, v.shape[0]))
        assert sum(c for _, _, c in step.local_ranges()) == sum(
            c for plan in step.plans for _, c in plan["slices"][r])
    views.sort()
    for a, b in zip(views, views[1:]):
        assert a[1] <= b[0]
    for g, (L, _, _) in enumerate(shapes):
        got = sorted((s, c) for _, _, gg, s, c in views if gg == g)
        cover = []
        for s, c in got:
            cover.extend(range(s, s + c))
        assert cover == list(range(L))


def test_auto_buckets_follow_the_model():
    """One rank needs no buckets; with more ranks the automatic fractions are
    positive, and their modelled step is no slower than a single bucket."""
    from polar_switch.distributed import (BUCKET_OVERHEAD_S, CIRCUIT_FLOPS_PER_S, GATHER_RECV_BYTES_PER_S,
                                          auto_bucket_fractions, simulate_buckets)
    banks = qwen3_0_6b_banks()
    assert auto_bucket_fractions(banks, 1, flops) == 1
    total = sum(L * flops(r, c) for L, r, c in banks)
    elems = sum(L * r * c for L, r, c in banks)
    for world in (2, 4, 8):
        fr = auto_bucket_fractions(banks, world, flops)
        fr = fr if isinstance(fr, list) else [1.0]
        assert all(f > 0 for f in fr)
        compute = total / world / CIRCUIT_FLOPS_PER_S
        gather = (world - 1) / world * elems * 2 / GATHER_RECV_BYTES_PER_S
        assert simulate_buckets(fr, compute, gather) <= simulate_buckets([1.0], compute, gather) + 1e-12
        # a schedule never ends before its transfer, nor before its compute
        t = simulate_buckets(fr, compute, gather)
        assert t >= gather and t >= compute + BUCKET_OVERHEAD_S


@pytest.mark.parametrize("counts,fractions", [([4, 7, 4, 7, 4], [1, 1, 1]), ([1, 0, 3], [1, 2]),
                                               ([28, 56], [1.0]), ([5, 2], [1, 2, 4, 8])])
def test_push_phase_ends(counts, fractions):
    """Cumulative per-phase counts: one list per input, as many entries as
    phases, non-decreasing, ending at the input's count, each phase about its
    fraction of the input."""
    from polar_switch.distributed import phase_ends
    ends = phase_ends(counts, fractions)
    assert len(ends) == len(counts)
    total = sum(fractions)
    for c, e in zip(counts, ends):
        assert len(e) == len(fractions) and e[-1] == c
        assert all(0 <= a <= b for a, b in zip([0] + e, e))
        acc = 0.0
        for f, v in zip(fractions, e):
            acc += f
            assert abs(v - c * acc / total) <= 1.0


def test_overlap_phase_ranges_cover_each_output_once():
    """The ranges the overlap transport copies after each phase flag tile the
    rank's segment exactly: every element once, in the phase that finishes it."""
    from polar_switch.distributed import phase_ends, phase_ranges
    shapes = [(4, 16, 8), (7, 8, 8), (1, 24, 16), (0, 8, 8)]
    shapes = [s for s in shapes if s[0]]
    for fr in ([1.0], [1, 1, 1], [1, 2, 4, 8]):
        ends = phase_ends([s[0] for s in shapes], fr)
        rng = phase_ranges(shapes, ends)
        assert len(rng) == len(fr)
        covered = []
        for k, r in enumerate(rng):
            for start, n in r:
                covered.extend(range(start, start + n))
        assert sorted(covered) == list(range(sum(c * r * q for c, r, q in shapes)))
        # the matrices of phase k of input i lie in phase k's ranges
        off = 0
        for (c, r, q), e in zip(shapes, ends):
            lo = 0
            for k, hi in enumerate(e):
                for m in range(lo, hi):
                    a = off + m * r * q
                    assert any(s0 <= a and a + r * q <= s0 + n for s0, n in rng[k])
                lo = hi
            off += c * r * q


def test_push_is_chosen_only_where_it_can_run():
    """transport="auto" picks the fused push only for a native CUDA circuit on
    more than one rank; the gloo tests' CPU ranks take the collective."""
    from polar_switch.distributed import push_phase_fractions
    from polar_switch.distributed import PUSH_MAX_WORLD
    assert push_phase_fractions(2) == [1.0] and len(push_phase_fractions(8)) == 3
    assert PUSH_MAX_WORLD >= 2
    step = ShardedOrthogonalizer([(4, 64, 32)], device=torch.device("cpu"), world_size=1, rank=0,
                                 grouped_fn=lambda i, o: None)
    assert step.transport == "none"
    with pytest.raises(ValueError):
        ShardedOrthogonalizer([(4, 64, 32)], device=torch.device("cpu"), world_size=1, rank=0,
                              grouped_fn=lambda i, o: None, transport="bogus")


class _OracleSplitOps:
    """CPU stand-ins for the split-matrix kernels (test infrastructure)."""

    @staticmethod
    def sumsq(X):
        return X.double().pow(2).sum(dim=(-2, -1))

    @staticmethod
    def scale_cast(X, sums, epsilon):
        if sums is None:
            return X.half()
        den = sums.sqrt().float().reshape(-1, 1, 1) + epsilon
        return (X.float() / den).half()

    @staticmethod
    def gram_f32(Xh):
        Xa = Xh.float()
        return Xa.mT @ Xa if Xh.shape[-2] > Xh.shape[-1] else Xa @ Xa.mT

    @staticmethod
    def square(A, C, out, alpha, beta, diag):
        from oracle import circuit as oc
        out.copy_(oc.square(A, C, alpha, beta, diag))
        return out

    @staticmethod
    def apply(X, B, tall, residual):
        from oracle import circuit as oc
        return oc.apply(X, B, tall, residual)


def _split_worker(rank, world, port, shapes, result_queue):
    try:
        import datetime
        import torch.distributed as dist
        from polar_switch.distributed import make_sharded_orthogonalizer
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
        g = torch.Generator().manual_seed(9)
        banks = [torch.randn(*s, generator=g) for s in shapes]
        step = make_sharded_orthogonalizer(shapes, method="PS2_55", device="cpu", world_size=world,
                                           rank=rank, transport="collective")
        step.ops = _OracleSplitOps
        step(banks)
        result_queue.put((rank, type(step).__name__, [f.clone() for f in step.gathered_banks()]))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        result_queue.put((rank, None, f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))


@pytest.mark.parametrize("world,shapes", [(2, [(1, 64, 256)]), (4, [(2, 384, 96)])])
def test_split_matrices_gloo_match_the_whole_circuit(world, shapes):
    """Fewer matrices than ranks: each matrix is cut along its long side, the
    partial sums of squares and partial Grams are all-reduced, and the gathered
    result matches the FP64 circuit on the whole matrix within the tolerance
    of the whole-matrix path (the partial FP32 Grams are summed in another
    order, so the bits differ from an unsplit evaluation)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_split_worker, args=(r, world, port, shapes, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, kind, res = q.get(timeout=180)
            results[rank] = (kind, res)
    finally:
        for p in procs:
            p.join(timeout=10)
            if p.is_alive():
                p.kill()
    from oracle import circuit as oc
    g = torch.Generator().manual_seed(9)
    banks = [torch.randn(*s, generator=g) for s in shapes]
    ref64 = [oc.run_circuit(b, coefficients.PS2_55, acc=torch.float64) for b in banks]
    ref32 = [oc.run_circuit(b, coefficients.PS2_55) for b in banks]
    for r in range(world):
        kind, res = results[r]
        assert not isinstance(res, str), res
        assert kind == "SplitOrthogonalizer"
        for got, e64, e32 in zip(res, ref64, ref32):
            assert got.shape == e64.shape
            floor = oc.relative_frobenius(e32, e64)
            assert oc.relative_frobenius(got, e64) <= max(5e-3, 1.5 * floor)
