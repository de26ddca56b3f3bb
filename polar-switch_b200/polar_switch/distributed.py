"""FLOP-balanced multi-GPU orthogonalization for a Muon step.

A Muon step orthogonalizes every 2-D hidden-layer update; the matrices are
independent, so the work shards by whole matrix (the reference's NanoGPT
optimizer shards banks of same-shape matrices matrix-granularly across ranks:
training/train_nanogpt.py:3983-4037, 4119-4218). Here

  * `plan_shards` splits each bank (L same-shape matrices) into one contiguous
    slice per rank, choosing the slice sizes by longest-processing-time-first
    on the per-matrix circuit FLOPs so every rank gets about the same work;
    the plan is a pure function of the shapes, so every rank computes the same
    plan without communication;
  * `plan_buckets` cuts the matrices into a few consecutive buckets of chosen
    cost fractions (`auto_bucket_fractions`), so the transfer of one bucket
    overlaps the next one's math;
  * `ShardedOrthogonalizer` runs each bucket's local slices as one grouped
    circuit whose FP16 results land directly in that bucket's packed segment
    of the receive buffer (the circuit rounds to FP16, so FP16 is lossless).
    Each finished segment then reaches the other ranks while the next bucket
    computes: by default every rank pushes it into every peer's receive
    buffer (symmetric memory) with peer-to-peer copies that run on the copy
    engines, leaving the SMs to the circuits; alternatively an asynchronous
    in-place all_gather_into_tensor of the group's backend. With one rank
    nothing is communicated. `step_host` runs a step from and to pinned host
    memory with the transfers overlapping the circuits; `capture` / `replay`
    record a step as a CUDA graph.
"""

import heapq

import torch
import torch.distributed as dist

from . import circuit_flops, coefficients, make_polynomial_orthogonalizer


def plan_shards(banks, world_size, flops_fn):
    """Split banks across ranks.

    Args:
        banks: list of (L, rows, cols), one per bank of same-shape matrices.
        world_size: number of ranks.
        flops_fn: flops_fn(rows, cols) -> cost of one matrix.

    Returns:
        slices[rank][bank] = (start, count): the contiguous matrices of that
        bank the rank orthogonalizes. Every matrix is assigned exactly once.
    """
    if world_size < 1:
        raise ValueError("world_size must be positive")
    counts = [[0] * len(banks) for _ in range(world_size)]
    # Largest matrices first; ties broken by bank index for determinism.
    order = sorted(range(len(banks)), key=lambda g: (-flops_fn(banks[g][1], banks[g][2]), g))
    heap = [(0.0, r) for r in range(world_size)]
    for g in order:
        L, rows, cols = banks[g]
        cost = flops_fn(rows, cols)
        for _ in range(L):
            load, r = heapq.heappop(heap)
            counts[r][g] += 1
            heapq.heappush(heap, (load + cost, r))
    slices = [[None] * len(banks) for _ in range(world_size)]
    for g in range(len(banks)):
        start = 0
        for r in range(world_size):
            slices[r][g] = (start, counts[r][g])
            start += counts[r][g]
    return slices


def plan_loads(banks, slices, flops_fn):
    """Per-rank total cost of a plan (for diagnostics and tests)."""
    return [sum(c * flops_fn(banks[g][1], banks[g][2]) for g, (_, c) in enumerate(rank))
            for rank in slices]


def plan_buckets(banks, buckets, flops_fn):
    """Split the matrices of all banks into consecutive buckets by cost.

    Args:
        banks: list of (L, rows, cols).
        buckets: number of buckets of about equal cost, or a list of cost
            fractions (normalised to sum 1), first bucket first.
        flops_fn: flops_fn(rows, cols) -> cost of one matrix.

    Returns:
        list of buckets, each a list of (bank, start, count) pieces covering
        consecutive matrices of a bank; every matrix is in exactly one piece.
        Empty buckets are dropped.
    """
    fracs = [1.0] * buckets if isinstance(buckets, int) else [float(f) for f in buckets]
    if not fracs or any(f <= 0 for f in fracs):
        raise ValueError("buckets must be a positive count or a list of positive fractions")
    total = sum(L * flops_fn(r, c) for L, r, c in banks)
    bounds, acc = [], 0.0
    for f in fracs:
        acc += f
        bounds.append(total * acc / sum(fracs))
    out = [[] for _ in fracs]
    k, done = 0, 0.0
    for g, (L, rows, cols) in enumerate(banks):
        cost = flops_fn(rows, cols)
        i = 0
        while i < L:
            # Matrices of this bank that still fit the current bucket (at least one).
            room = bounds[k] - done
            take = L - i if k == len(fracs) - 1 else max(1, min(L - i, int(room / cost + 0.5)))
            out[k].append((g, i, take))
            i += take
            done += take * cost
            if k < len(fracs) - 1 and done >= bounds[k] - 0.5 * cost:
                k += 1
    return [b for b in out if b]


# Rates used only to shape the buckets: the whole-step circuit rate of one
# B200 on n ~ 1024 matrices, the rate at which a GPU receives the gathered
# updates over NVLink (copy-engine pushes: ~0.7 TB/s at 2 and 8 GPUs), and the
# fixed cost of running a bucket as its own circuit (launch tails of its
# ~40 kernels), all measured on B200.
CIRCUIT_FLOPS_PER_S = 7.5e14
GATHER_RECV_BYTES_PER_S = 7.0e11
BUCKET_OVERHEAD_S = 2.0e-4


def simulate_buckets(fractions, compute_s, gather_s, overhead_s=BUCKET_OVERHEAD_S):
    """Modelled step time of a bucket schedule: the circuits run back to back on
    one stream, each bucket's gather starts when its circuits and the previous
    gather are done."""
    total = float(sum(fractions))
    t_compute = t_gather = 0.0
    for f in fractions:
        t_compute += overhead_s + compute_s * f / total
        t_gather = max(t_gather, t_compute) + gather_s * f / total
    return t_gather


def phase_ends(counts, fractions):
    """Cumulative per-phase matrix counts of each input for a push launch.

    counts: matrices of each input; fractions: relative phase sizes. Returns
    one list per input, non-decreasing, ending at its count (phases may be
    empty for small inputs)."""
    total = float(sum(fractions))
    cum, acc = [], 0.0
    for f in fractions:
        acc += f
        cum.append(acc / total)
    out = []
    for c in counts:
        e = [min(c, max(0, int(round(c * x)))) for x in cum]
        e[-1] = c
        for j in range(1, len(e)):
            e[j] = max(e[j], e[j - 1])
        out.append(e)
    return out


def phase_ranges(shapes, ends):
    """Per phase, the (start, length) element ranges of a segment that packs
    inputs of `shapes` ((count, rows, cols) each) one after another, covering
    the matrices each phase completes (`ends` from phase_ends); adjacent
    ranges are merged."""
    out = [[] for _ in (ends[0] if ends else [])]
    off = 0
    for (count, rows, cols), e in zip(shapes, ends):
        per = rows * cols
        lo = 0
        for k, hi in enumerate(e):
            if hi > lo:
                rng = out[k]
                start, n = off + lo * per, (hi - lo) * per
                if rng and rng[-1][0] + rng[-1][1] == start:
                    rng[-1] = (rng[-1][0], rng[-1][1] + n)
                else:
                    rng.append((start, n))
            lo = hi
        off += count * per
    return out


# Push transport: phases of the rank's matrices inside its one launch. With
# two ranks the step is compute-bound (each GPU receives half the updates
# while computing the other half) and one phase is best; from four ranks on
# the NVLink receive time exceeds the circuits and three equal phases put the
# first results on the links early (modelled on the whole-circuit kernel's
# schedule and measured on B200).
# Largest group for which "auto" picks the push transport. The SM-issued
# stores reach the peers more slowly than the copy engines (Qwen step on B200,
# push against copy engines: 3.21 vs 3.30 ms at 2 GPUs, where the transfer
# hides under the circuits; 2.50 vs 2.25 ms at 4 and 2.40 vs 1.98 ms at 8).
PUSH_MAX_WORLD = 2

# Phases of the "overlap" transport's launch: shrinking shares of each bank,
# so the last phase's push, exposed after the launch, is small (4 GPUs, Qwen
# step: 2.22 ms against 2.42 with four equal phases).
OVERLAP_PHASES = [3.0, 3.0, 2.0, 1.0, 0.5]


def push_phase_fractions(world_size):
    return [1.0] if world_size <= 2 else [1.0, 1.0, 1.0]


def auto_bucket_fractions(banks, world_size, flops_fn):
    """Bucket cost fractions for overlapping the gather with the circuits.

    Candidates are geometric schedules (fractions proportional to r**k, k <
    count): r < 1 front-loads the work, so a compute-bound step exposes only a
    small last gather; r > 1 starts a gather-bound step's transfers early. The
    candidate with the least modelled step time (`simulate_buckets`) wins.
    """
    flops = sum(L * flops_fn(r, c) for L, r, c in banks)
    elems = sum(L * r * c for L, r, c in banks)
    if world_size < 2 or flops <= 0:
        return 1
    compute_s = flops / world_size / CIRCUIT_FLOPS_PER_S
    gather_s = (world_size - 1) / world_size * elems * 2 / GATHER_RECV_BYTES_PER_S
    if gather_s > compute_s:
        # Transfer-bound: a growing schedule, so the first push starts after a
        # small first bucket. On 8 B200s (Qwen step) 53 + 70 + 73 matrices
        # measured 1.73 ms against 1.95 ms for the shrinking 108 + 52 + 36 the
        # model preferred (it does not see the barrier and copy start latencies).
        return [1.0, 1.4, 1.96]
    best = ([1.0], simulate_buckets([1.0], compute_s, gather_s))
    for count in (2, 3, 4, 5):
        for r in (0.2, 0.25, 1 / 3, 0.5, 0.7, 1.0, 1.4, 2.0, 3.0):
            fr = [r ** k for k in range(count)]
            t = simulate_buckets(fr, compute_s, gather_s)
            if t < best[1] * (1 - 1e-9):
                best = (fr, t)
    return best[0]


class ShardedOrthogonalizer:
    """Orthogonalize banks of matrices across the ranks of a process group.

    Every rank passes the same list of banks (CUDA tensors (L_g, rows_g,
    cols_g), e.g. momentum buffers after gradient averaging). The matrices are
    cut into buckets of consecutive matrices (`plan_buckets`); each bucket is
    split across the ranks by `plan_shards`, orthogonalized as one grouped
    circuit, and its FP16 results are all-gathered asynchronously while the
    next bucket computes. ``__call__`` returns the gathered buffer (stream-
    ordered); ``bank_updates`` gives, per bank, the (start, view) slices of it.
    """

    def __init__(self, bank_shapes, method="PS2_55", epsilon=1e-7, group=None, device=None,
                 world_size=None, rank=None, grouped_fn=None, buckets=None, gemm_ctas=None,
                 transport="auto"):
        """``grouped_fn(inputs, outs)`` replaces the B200 grouped circuit (used by
        the CPU tests of the sharding logic); by default the circuit runs on
        the GPU. ``buckets``: number of buckets or their cost fractions; by
        default 1 on one rank and `auto_bucket_fractions` otherwise. ``gemm_ctas``: cap on the CTAs of the GEMM
        grids while a gather may be in flight, leaving SMs to the collective
        (None = no cap). ``transport``: how a bucket reaches the other ranks:
        "copy_engine" (each rank pushes its segment into every peer's receive
        buffer, a symmetric-memory allocation, with peer-to-peer copies that
        run on the copy engines and leave every SM to the circuits),
        "collective" (an asynchronous all_gather_into_tensor of the group's
        backend), "push" (one launch per rank for all its matrices, whose last
        apply stores every result tile into every peer's receive buffer as it
        is computed: the gather fused into the circuit; ``buckets`` then
        give the phases the launch schedules one after another, by default
        `push_phase_fractions`) or "auto" (push on CUDA for groups of up to
        PUSH_MAX_WORLD ranks when the rank's work fits one whole-circuit
        launch, else copy engines; the collective off CUDA)."""
        self.group = group
        if world_size is None:
            world_size = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        if rank is None:
            rank = dist.get_rank(group) if world_size > 1 else 0
        self.world_size, self.rank = world_size, rank
        self.polar = make_polynomial_orthogonalizer(method, epsilon=epsilon)
        self.native_circuit = grouped_fn is None
        self.grouped_fn = grouped_fn or (lambda inputs, outs: self.polar.grouped(inputs, outs=outs))
        self.gemm_ctas = gemm_ctas
        table = self.polar.table
        self.flops_fn = lambda r, c: circuit_flops(table, r, c)
        self.bank_shapes = [tuple(int(v) for v in s) for s in bank_shapes]
        if transport not in ("auto", "copy_engine", "collective", "push", "overlap"):
            raise ValueError(f"unknown transport {transport!r}")
        if (transport == "auto" and 1 < world_size <= PUSH_MAX_WORLD and self.native_circuit
                and torch.device(device if device is not None else "cuda").type == "cuda"
                and self._push_fits()):
            transport = "push"
        self.phase_fractions = None
        if transport == "push":
            self.phase_fractions = (push_phase_fractions(world_size) if buckets is None else
                                    [1.0] * buckets if isinstance(buckets, int) else list(buckets))
            buckets = 1
        elif transport == "overlap":
            self.phase_fractions = (list(OVERLAP_PHASES) if buckets is None else
                                    [1.0] * buckets if isinstance(buckets, int) else list(buckets))
            buckets = 1
        if buckets is None:
            buckets = 1 if world_size == 1 else auto_bucket_fractions(self.bank_shapes, world_size,
                                                                       self.flops_fn)
        self.buckets = plan_buckets(self.bank_shapes, buckets, self.flops_fn)
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        # Per bucket: the sub-banks it holds, their split across ranks and the
        # padded per-rank segment length. Segments are padded to a multiple of
        # 128 elements (256 B) so the per-problem outputs stay 16-byte aligned.
        self.plans = []
        offset = 0
        for pieces in self.buckets:
            shapes = [(count, self.bank_shapes[g][1], self.bank_shapes[g][2]) for g, _, count in pieces]
            slices = plan_shards(shapes, world_size, self.flops_fn)
            elems = [sum(c * r * k for (_, c), (_, r, k) in zip(rs, shapes)) for rs in slices]
            seg = max(max(-(-e // 128) * 128 for e in elems), 128)
            self.plans.append({"pieces": pieces, "slices": slices, "seg": seg, "offset": offset})
            offset += world_size * seg
        # In-place gathers: this rank's segment of each bucket's receive region
        # is its send buffer, so the circuit writes results where they end up.
        if transport == "auto":
            transport = "copy_engine" if world_size > 1 and self.device.type == "cuda" else "collective"
        if world_size == 1:
            transport = "none"
        self.transport = transport
        numel = max(offset, 1)
        if transport in ("copy_engine", "push", "overlap"):
            import torch.distributed._symmetric_memory as symm
            self.recv = symm.empty(numel, device=self.device, dtype=torch.float16)
            handle = symm.rendezvous(self.recv, self.group if self.group is not None else dist.group.WORLD)
            self._peer_recv = [handle.get_buffer(p, (numel,), torch.float16) for p in range(world_size)]
            self._handle = handle
            self._comm = torch.cuda.Stream(device=self.device)
            self._flag = torch.zeros(1, device=self.device, dtype=torch.int32)
            self._push_unsupported = False
            if transport == "overlap":
                plan = self.plans[0]
                views = self._segment_views(plan, rank)
                ends = phase_ends([v.shape[0] for _, _, v in views], self.phase_fractions)
                self._signal = {"flags": torch.zeros(2 * len(self.phase_fractions) + 1, device=self.device,
                                                     dtype=torch.int32), "phase_ends": ends}
                self._phase_ranges = phase_ranges([tuple(v.shape) for _, _, v in views], ends)
            if transport == "push":
                plan = self.plans[0]
                counts = [v.shape[0] for _, _, v in self._segment_views(plan, self.rank)]
                self._push = {"local": self.recv.data_ptr(),
                              "peers": [self._peer_recv[p].data_ptr() for p in range(world_size)
                                        if p != rank],
                              "phase_ends": phase_ends(counts, self.phase_fractions)}
        else:
            self.recv = torch.empty(numel, device=self.device, dtype=torch.float16)
        self.flops_total = sum(L * self.flops_fn(r, c) for L, r, c in self.bank_shapes)
        self.flops_per_rank = [0.0] * world_size
        for plan in self.plans:
            shapes = [(c, self.bank_shapes[g][1], self.bank_shapes[g][2]) for g, _, c in plan["pieces"]]
            for r, load in enumerate(plan_loads(shapes, plan["slices"], self.flops_fn)):
                self.flops_per_rank[r] += load

    def _push_fits(self):
        """Whether every rank's share fits one whole-circuit launch (at most 8
        problems: one per bank with matrices on the rank, all unpadded)."""
        if len(self.bank_shapes) > 8:
            return False
        return all(r % 8 == 0 and c % 8 == 0 for _, r, c in self.bank_shapes)

    def _region(self, plan):
        return self.recv[plan["offset"]:plan["offset"] + self.world_size * plan["seg"]]

    def _segment(self, plan, rank):
        base = plan["offset"] + rank * plan["seg"]
        return self.recv[base:base + plan["seg"]]

    def _segment_views(self, plan, rank):
        """(bank, start within the bank, view) for each non-empty slice of one
        rank's segment of a bucket."""
        views, off = [], 0
        seg = self._segment(plan, rank)
        for (g, base, _), (start, count) in zip(plan["pieces"], plan["slices"][rank]):
            if count:
                rows, cols = self.bank_shapes[g][1:]
                n = count * rows * cols
                views.append((g, base + start, seg[off:off + n].view(count, rows, cols)))
                off += n
        return views

    def local_ranges(self, rank=None):
        """(bank, start, count) of every matrix range the given rank orthogonalizes."""
        rank = self.rank if rank is None else rank
        return [(g, start, v.shape[0]) for plan in self.plans for g, start, v in self._segment_views(plan, rank)]

    def _check(self, banks):
        if len(banks) != len(self.bank_shapes):
            raise ValueError("expected one tensor per bank")
        for X, shape in zip(banks, self.bank_shapes):
            if tuple(X.shape) != shape:
                raise ValueError(f"bank shape {tuple(X.shape)} does not match the plan {shape}")

    def _compute_bucket(self, banks, plan, push=None, signal=None):
        ready = getattr(self, "_input_events", None)
        if ready is not None:  # inputs of this bucket still arriving from the host
            torch.cuda.current_stream(self.device).wait_event(ready[id(plan)])
        inputs, outputs = [], []
        for g, start, view in self._segment_views(plan, self.rank):
            inputs.append(banks[g][start:start + view.shape[0]])
            outputs.append(view)
        if inputs:
            if signal is not None:
                self.polar.grouped(inputs, outs=outputs, signal=signal)
            elif push is not None:
                self.polar.grouped(inputs, outs=outputs, push=push)
            else:
                self.grouped_fn(inputs, outputs)

    def compute_local(self, banks):
        """Orthogonalize this rank's slices into its segments (no communication)."""
        self._check(banks)
        for plan in self.plans:
            self._compute_bucket(banks, plan)
        return self.recv

    def __call__(self, banks):
        """Orthogonalize all banks across the group; returns the gathered FP16
        buffer (ready in the order of the current stream)."""
        self._check(banks)
        if self.world_size == 1:
            return self.compute_local(banks)
        cap = self.native_circuit and self.gemm_ctas
        if cap:
            from . import _native
            previous = _native.set_max_ctas(self.gemm_ctas)
        try:
            if self.transport == "copy_engine":
                self._step_copy_engine(banks)
            elif self.transport == "push":
                self._step_push(banks)
            elif self.transport == "overlap":
                self._step_overlap(banks)
            else:
                self._step_collective(banks)
        finally:
            if cap:
                _native.set_max_ctas(previous)
        return self.recv

    def _step_collective(self, banks):
        works = []
        try:
            for plan in self.plans:
                self._compute_bucket(banks, plan)
                works.append(dist.all_gather_into_tensor(self._region(plan), self._segment(plan, self.rank),
                                                         group=self.group, async_op=True))
        finally:
            for w in works:
                w.wait()

    def _barrier_on(self, stream):
        """A group-wide barrier ordered on `stream` (a one-element all-reduce)."""
        with torch.cuda.stream(stream):
            dist.all_reduce(self._flag, group=self.group)

    def _step_copy_engine(self, banks):
        """Push each finished bucket into every peer's receive buffer from a side
        stream while the next bucket computes on the current stream.

        Ordering: a barrier on the current stream before the first circuit, which
        the side stream waits for, so no peer still reads the previous step's
        results when the first push lands; after the last push a second
        barrier (on the side stream) tells every rank
        that all pushes into its buffer are complete, and the current stream
        waits for it."""
        main = torch.cuda.current_stream(self.device)
        comm = self._comm
        # The first barrier runs on the caller's stream before any circuit:
        # issued on the side stream, its collective kernel could find every SM
        # held by the first persistent circuit launch and hold back the pushes.
        self._barrier_on(main)
        comm.wait_stream(main)
        order = [(self.rank + i) % self.world_size for i in range(1, self.world_size)]
        for plan in self.plans:
            self._compute_bucket(banks, plan)
            comm.wait_stream(main)
            base = plan["offset"] + self.rank * plan["seg"]
            src = self.recv[base:base + plan["seg"]]
            with torch.cuda.stream(comm):
                for p in order:
                    self._peer_recv[p][base:base + plan["seg"]].copy_(src, non_blocking=True)
        self._barrier_on(comm)
        main.wait_stream(comm)

    def _step_push(self, banks):
        """One launch per rank computes its matrices and stores every result
        tile into every peer's receive buffer as it is computed. A barrier on
        the current stream before the launch (no peer still reads the
        previous step's results) and one after it (every peer's launch, and
        so every store into this rank's buffer, has completed) order it."""
        from . import _native
        main = torch.cuda.current_stream(self.device)
        plan = self.plans[0]
        self._barrier_on(main)
        if not self._push_unsupported:
            try:
                self._compute_bucket(banks, plan, push=self._push)
            except _native.NativeError as e:
                # Refused before anything ran (shapes or table outside one
                # whole-circuit launch; the same on every rank): from now on
                # compute, then copy the segment to the peers. The collective
                # steps stay the same on every rank.
                if e.code != _native.PS_ERR_UNSUPPORTED:
                    raise
                self._push_unsupported = True
        if self._push_unsupported:
            self._compute_bucket(banks, plan)
            base = plan["offset"] + self.rank * plan["seg"]
            src = self.recv[base:base + plan["seg"]]
            for p in range(self.world_size):
                if p != self.rank:
                    self._peer_recv[p][base:base + plan["seg"]].copy_(src, non_blocking=True)
        self._barrier_on(main)

    def _step_overlap(self, banks):
        """One launch per rank computes its matrices phase by phase and raises a
        device flag as each phase's results are stored; a side stream waits on
        each flag (ps_stream_wait_flag) and pushes that phase's part of the
        segment into every peer's receive buffer with copy-engine copies while
        the launch computes the next phases. Barriers as in the copy-engine
        step: before the first push (no peer still reads the previous results)
        and after the last (every push into this rank's buffer is complete)."""
        from . import _native
        main = torch.cuda.current_stream(self.device)
        comm = self._comm
        plan = self.plans[0]
        flags = self._signal["flags"]
        flags.zero_()                      # before the launch and before the waits
        # first barrier on the caller's stream, before the persistent launch
        # takes every SM (on the side stream it would wait for that launch)
        self._barrier_on(main)
        comm.wait_stream(main)
        base = plan["offset"] + self.rank * plan["seg"]
        order = [(self.rank + i) % self.world_size for i in range(1, self.world_size)]
        if not self._push_unsupported:
            try:
                self._compute_bucket(banks, plan, signal=self._signal)
            except _native.NativeError as e:
                if e.code != _native.PS_ERR_UNSUPPORTED:
                    raise
                self._push_unsupported = True
        if self._push_unsupported:  # refused before anything ran: compute, then copy it all
            self._compute_bucket(banks, plan)
            comm.wait_stream(main)
            ranges = [[(0, plan["seg"])]]
        else:
            ranges = self._phase_ranges
        with torch.cuda.stream(comm):
            for k, rng in enumerate(ranges):
                # a phase with results here was launched: its flag is raised
                # by the launch at the latest when it exits
                if rng and not self._push_unsupported:
                    _native.stream_wait_flag(comm, flags.data_ptr() + 4 * k, 1)
                for start, n in rng:
                    src = self.recv[base + start:base + start + n]
                    for p in order:
                        self._peer_recv[p][base + start:base + start + n].copy_(src, non_blocking=True)
        self._barrier_on(comm)
        main.wait_stream(comm)

    def step_host(self, host_banks, host_out=None):
        """One step from host memory: copies this rank's slices of `host_banks`
        (pinned CPU tensors shaped like the plan) to the device bucket by bucket
        on a copy stream, computes each bucket as soon as its inputs are there,
        and copies the gathered FP16 result back into `host_out` (a pinned FP16
        tensor of `recv`'s size; allocated when None) -- with one rank bucket by
        bucket as each finishes, with several once the exchange is complete.
        Transfers in both directions overlap the circuits. Returns `host_out`,
        valid once the caller's current stream has reached this point."""
        if self.device.type != "cuda":
            raise ValueError("step_host needs a CUDA device")
        self._check(host_banks)
        dev = self.device
        if getattr(self, "_dev_in", None) is None:
            self._dev_in = [torch.empty(b.shape, dtype=b.dtype, device=dev) for b in host_banks]
            self._h2d = torch.cuda.Stream(device=dev)
            self._d2h = torch.cuda.Stream(device=dev)
        if host_out is None:
            host_out = torch.empty(self.recv.numel(), dtype=torch.float16, pin_memory=True)
        main = torch.cuda.current_stream(dev)
        self._h2d.wait_stream(main)  # the staging buffers are free again
        events = {}
        with torch.cuda.stream(self._h2d):
            for plan in self.plans:
                for g, start, view in self._segment_views(plan, self.rank):
                    n = view.shape[0]
                    self._dev_in[g][start:start + n].copy_(host_banks[g][start:start + n], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self._h2d)
                events[id(plan)] = ev
        self._input_events = events
        try:
            if self.world_size == 1:
                for plan in self.plans:
                    self._compute_bucket(self._dev_in, plan)
                    self._d2h.wait_stream(main)
                    region = self._region(plan)
                    with torch.cuda.stream(self._d2h):
                        host_out[plan["offset"]:plan["offset"] + region.numel()].copy_(region, non_blocking=True)
            else:
                self(self._dev_in)
                self._d2h.wait_stream(main)
                with torch.cuda.stream(self._d2h):
                    host_out.copy_(self.recv, non_blocking=True)
        finally:
            self._input_events = None
        main.wait_stream(self._d2h)
        main.wait_stream(self._h2d)
        return host_out

    def capture(self, banks, warmup=2):
        """Record one whole step on these bank tensors as a CUDA graph (after
        `warmup` eager steps); `replay()` then runs it again with no host work
        per launch. The banks must stay at the same addresses (e.g. persistent
        momentum buffers)."""
        if self.device.type != "cuda":
            raise ValueError("graph capture needs CUDA tensors")
        for _ in range(warmup):
            self(banks)
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self(banks)
        torch.cuda.synchronize(self.device)
        self._graph = graph
        return graph

    def replay(self):
        """Run the captured step; returns the gathered buffer (stream-ordered)."""
        self._graph.replay()
        return self.recv

    def close(self):
        """Drop the peer mappings of the receive buffer (before the process
        group is destroyed)."""
        for name in ("_graph", "_peer_recv", "_handle", "_dev_in"):
            if hasattr(self, name):
                delattr(self, name)

    def bank_updates(self):
        """Per bank, the list of (start, FP16 view) slices of the gathered result."""
        out = [[] for _ in self.bank_shapes]
        for plan in self.plans:
            for r in range(self.world_size):
                for g, start, view in self._segment_views(plan, r):
                    out[g].append((start, view))
        return out

    def gathered_banks(self):
        """The full update of every bank as one FP16 tensor each (copies)."""
        res = []
        for g, parts in enumerate(self.bank_updates()):
            parts.sort(key=lambda p: p[0])
            res.append(torch.cat([v for _, v in parts]) if parts else None)
        return res


def split_plan(bank_shapes, world_size):
    """Whether and how to split matrices across ranks: with fewer matrices than
    ranks (the 4 x 8192 x 28672 stress batch on 8 GPUs), whole-matrix shards
    would leave ranks idle, so each matrix is cut along its long dimension into
    world_size / M parts, one per rank. Returns None (shard whole matrices) or
    (parts per matrix, part length), the length a multiple of 8."""
    M = sum(L for L, _, _ in bank_shapes)
    if world_size < 2 or M >= world_size or world_size % M:
        return None
    parts = world_size // M
    longest = max(max(r, c) for _, r, c in bank_shapes)
    if any(max(r, c) != longest for _, r, c in bank_shapes):
        return None  # one part length for every matrix keeps the plan simple
    if any(r % 8 or c % 8 for _, r, c in bank_shapes):
        return None  # parts of whole 16-byte rows, no padding
    length = -(-(-(-longest // parts)) // 8) * 8
    last = longest - (parts - 1) * length
    for _, r, c in bank_shapes:
        n = min(r, c)
        # every part keeps the matrix's orientation (tall parts stay taller
        # than wide, wide parts at least square), so the kernels treat a part
        # exactly like the whole matrix
        if last <= 0 or (r > c and last <= n) or (r <= c and last < n):
            return None
    return parts, length


class SplitOrthogonalizer:
    """Orthogonalize fewer matrices than ranks: each matrix is cut along its
    long dimension (columns of a wide matrix, rows of a tall one) into one part
    per rank of its group. Per outer iteration the ranks of a group sum their
    partial FP32 Grams (an all-reduce of n x n, the one exchange step), round
    once to FP16, run the inner iterations on the replicated n x n buffers and
    apply them to their own part; the normalisation sums the parts' sums of
    squares the same way. The result parts are then gathered like whole
    matrices. Same interface as ShardedOrthogonalizer.

    ``ops`` supplies sumsq / scale_cast / gram_f32 / square / apply (default:
    the B200 kernels of polar_switch.cuda_ops; the CPU tests pass an oracle).
    """

    def __init__(self, bank_shapes, method="PS2_55", epsilon=1e-7, group=None, device=None,
                 world_size=None, rank=None, ops=None, transport="auto"):
        if world_size is None:
            world_size = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        if rank is None:
            rank = dist.get_rank(group) if world_size > 1 else 0
        self.world_size, self.rank, self.group = world_size, rank, group
        self.bank_shapes = [tuple(int(v) for v in s) for s in bank_shapes]
        plan = split_plan(self.bank_shapes, world_size)
        if plan is None:
            raise ValueError("these banks do not split evenly across the ranks")
        self.parts, self.length = plan
        self.polar = make_polynomial_orthogonalizer(method, epsilon=epsilon)
        self.table, self.epsilon = self.polar.table, epsilon
        if ops is None:
            from . import cuda_ops as ops
        self.ops = ops
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.matrices = [(g, i) for g, (L, _, _) in enumerate(self.bank_shapes) for i in range(L)]
        self.matrix = rank // self.parts
        self.part = rank % self.parts
        # One process group per matrix; every rank creates all of them, in order.
        self.groups = []
        for m in range(len(self.matrices)):
            ranks = list(range(m * self.parts, (m + 1) * self.parts))
            self.groups.append(dist.new_group(ranks) if world_size > 1 else None)
        g, _ = self.matrices[self.matrix]
        _, rows, cols = self.bank_shapes[g]
        self.tall = rows > cols
        self.n = min(rows, cols)
        lo = self.part * self.length
        hi = min(max(rows, cols), lo + self.length)
        self.span = (lo, hi)
        seg = self.n * self.length
        self.seg = -(-seg // 128) * 128
        if transport == "auto":
            transport = "collective"
        if transport != "collective":
            raise ValueError("split matrices are gathered with the collective transport")
        self.transport = transport
        self.recv = torch.empty(world_size * self.seg, device=self.device, dtype=torch.float16)
        table = self.table
        self.flops_total = sum(L * circuit_flops(table, r, c) for L, r, c in self.bank_shapes)
        self.plans = [{"pieces": [], "seg": self.seg, "offset": 0}]

    def _part_view(self, X, part, tall):
        lo = part * self.length
        hi = min(X.shape[-2] if tall else X.shape[-1], lo + self.length)
        return X[lo:hi, :] if tall else X[:, lo:hi]

    def _check(self, banks):
        if len(banks) != len(self.bank_shapes):
            raise ValueError("expected one tensor per bank")
        for X, shape in zip(banks, self.bank_shapes):
            if tuple(X.shape) != shape:
                raise ValueError(f"bank shape {tuple(X.shape)} does not match the plan {shape}")

    def compute_local(self, banks):
        """Orthogonalize this rank's part of its matrix into its segment of recv."""
        ops, grp = self.ops, self.groups[self.matrix]
        g, i = self.matrices[self.matrix]
        Xj = self._part_view(banks[g][i], self.part, self.tall)
        sums = ops.sumsq(Xj[None])
        if self.world_size > 1:
            dist.all_reduce(sums, group=grp)
        Xh = ops.scale_cast(Xj[None], sums, self.epsilon)
        n = self.n
        buffers = 1 + max(max(w, s, a) for _, steps in self.table for w, s, a, *_ in steps)
        work = [torch.empty((1, n, n), device=Xh.device, dtype=torch.float16) for _ in range(buffers)]
        for residual, steps in self.table:
            G = ops.gram_f32(Xh)
            if self.world_size > 1:
                dist.all_reduce(G, group=grp)
            work[0] = ops.scale_cast(G, None, 0.0)
            for dst, src, add, alpha, beta, diag in steps:
                ops.square(work[src], work[add], work[dst], alpha, beta, diag)
            Xh = ops.apply(Xh, work[steps[-1][0]], self.tall, residual)
        flat = Xh.reshape(-1)
        self.recv[self.rank * self.seg:self.rank * self.seg + flat.numel()].copy_(flat)
        return self.recv

    def __call__(self, banks):
        """Orthogonalize all banks across the group; returns the gathered FP16 buffer."""
        self._check(banks)
        self.compute_local(banks)
        if self.world_size > 1:
            dist.all_gather_into_tensor(self.recv, self.recv[self.rank * self.seg:(self.rank + 1) * self.seg],
                                        group=self.group)
        return self.recv

    def local_ranges(self, rank=None):
        """(bank, start, count) of the matrix whose part the rank orthogonalizes."""
        rank = self.rank if rank is None else rank
        g, i = self.matrices[rank // self.parts]
        return [(g, i, 1)]

    def gathered_banks(self):
        """The full update of every bank as one FP16 tensor each (copies)."""
        out = []
        for g, (L, rows, cols) in enumerate(self.bank_shapes):
            mats = []
            for i in range(L):
                m = self.matrices.index((g, i))
                pieces = []
                for part in range(self.parts):
                    r = m * self.parts + part
                    lo = part * self.length
                    hi = min(max(rows, cols), lo + self.length)
                    shape = (hi - lo, cols) if rows > cols else (rows, hi - lo)
                    n_el = shape[0] * shape[1]
                    pieces.append(self.recv[r * self.seg:r * self.seg + n_el].view(shape))
                mats.append(torch.cat(pieces, dim=0 if rows > cols else 1))
            out.append(torch.stack(mats))
        return out

    def _step_push(self, banks):
        """One launch per rank computes its matrices and stores every result
        tile into every peer's receive buffer as it is computed. A barrier on
        the current stream before the launch (no peer still reads the
        previous step's results) and one after it (every peer's launch, and
        so every store into this rank's buffer, has completed) order it."""
        from . import _native
        main = torch.cuda.current_stream(self.device)
        plan = self.plans[0]
        self._barrier_on(main)
        if not self._push_unsupported:
            try:
                self._compute_bucket(banks, plan, push=self._push)
            except _native.NativeError as e:
                # Refused before anything ran (shapes or table outside one
                # whole-circuit launch; the same on every rank): from now on
                # compute, then copy the segment to the peers. The collective
                # steps stay the same on every rank.
                if e.code != _native.PS_ERR_UNSUPPORTED:
                    raise
                self._push_unsupported = True
        if self._push_unsupported:
            self._compute_bucket(banks, plan)
            base = plan["offset"] + self.rank * plan["seg"]
            src = self.recv[base:base + plan["seg"]]
            for p in range(self.world_size):
                if p != self.rank:
                    self._peer_recv[p][base:base + plan["seg"]].copy_(src, non_blocking=True)
        self._barrier_on(main)

    def _step_overlap(self, banks):
        """One launch per rank computes its matrices phase by phase and raises a
        device flag as each phase's results are stored; a side stream waits on
        each flag (ps_stream_wait_flag) and pushes that phase's part of the
        segment into every peer's receive buffer with copy-engine copies while
        the launch computes the next phases. Barriers as in the copy-engine
        step: before the first push (no peer still reads the previous results)
        and after the last (every push into this rank's buffer is complete)."""
        from . import _native
        main = torch.cuda.current_stream(self.device)
        comm = self._comm
        plan = self.plans[0]
        flags = self._signal["flags"]
        flags.zero_()                      # before the launch and before the waits
        # first barrier on the caller's stream, before the persistent launch
        # takes every SM (on the side stream it would wait for that launch)
        self._barrier_on(main)
        comm.wait_stream(main)
        base = plan["offset"] + self.rank * plan["seg"]
        order = [(self.rank + i) % self.world_size for i in range(1, self.world_size)]
        if not self._push_unsupported:
            try:
                self._compute_bucket(banks, plan, signal=self._signal)
            except _native.NativeError as e:
                if e.code != _native.PS_ERR_UNSUPPORTED:
                    raise
                self._push_unsupported = True
        if self._push_unsupported:  # refused before anything ran: compute, then copy it all
            self._compute_bucket(banks, plan)
            comm.wait_stream(main)
            ranges = [[(0, plan["seg"])]]
        else:
            ranges = self._phase_ranges
        with torch.cuda.stream(comm):
            for k, rng in enumerate(ranges):
                # a phase with results here was launched: its flag is raised
                # by the launch at the latest when it exits
                if rng and not self._push_unsupported:
                    _native.stream_wait_flag(comm, flags.data_ptr() + 4 * k, 1)
                for start, n in rng:
                    src = self.recv[base + start:base + start + n]
                    for p in order:
                        self._peer_recv[p][base + start:base + start + n].copy_(src, non_blocking=True)
        self._barrier_on(comm)
        main.wait_stream(comm)

    def step_host(self, host_banks, host_out=None):
        """One step from pinned host banks: uploads this rank's matrix, computes
        its part and downloads the gathered FP16 buffer into `host_out`."""
        self._check(host_banks)
        if getattr(self, "_dev_in", None) is None:
            self._dev_in = [torch.empty(b.shape, dtype=b.dtype, device=self.device) for b in host_banks]
        if host_out is None:
            host_out = torch.empty(self.recv.numel(), dtype=torch.float16, pin_memory=True)
        g, i = self.matrices[self.matrix]
        self._dev_in[g][i].copy_(host_banks[g][i], non_blocking=True)
        self(self._dev_in)
        host_out.copy_(self.recv, non_blocking=True)
        return host_out

    def capture(self, banks, warmup=2):
        """Record one step as a CUDA graph (see ShardedOrthogonalizer.capture)."""
        for _ in range(warmup):
            self(banks)
        torch.cuda.synchronize(self.device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self(banks)
        torch.cuda.synchronize(self.device)
        self._graph = graph
        return graph

    def replay(self):
        self._graph.replay()
        return self.recv

    def close(self):
        for name in ("_graph", "_dev_in"):
            if hasattr(self, name):
                delattr(self, name)


def make_sharded_orthogonalizer(bank_shapes, **kwargs):
    """ShardedOrthogonalizer, or SplitOrthogonalizer when there are fewer
    matrices than ranks and they split evenly (`split_plan`)."""
    world = kwargs.get("world_size")
    if world is None:
        world = dist.get_world_size(kwargs.get("group")) if dist.is_available() and dist.is_initialized() else 1
    if split_plan([tuple(int(v) for v in s) for s in bank_shapes], world) is not None:
        keep = {k: v for k, v in kwargs.items()
                if k in ("method", "epsilon", "group", "device", "world_size", "rank", "transport")}
        if keep.get("transport") == "copy_engine":
            keep["transport"] = "collective"
        return SplitOrthogonalizer(bank_shapes, **keep)
    return ShardedOrthogonalizer(bank_shapes, **kwargs)


def qwen3_0_6b_banks(layers=28, hidden=1024):
    """Bank shapes of a Qwen3-0.6B Muon step (training/configs/qwen600m.json:26-34)."""
    inter = 3 * hidden
    return [(layers, 2 * hidden, hidden),       # q_proj (tall)
            (2 * layers, hidden, hidden),       # k_proj, v_proj
            (layers, hidden, 2 * hidden),       # o_proj (wide)
            (2 * layers, inter, hidden),        # gate_proj, up_proj (tall)
            (layers, hidden, inter)]            # down_proj (wide)


def gemma3_1b_banks(layers=26, hidden=1152):
    """Bank shapes of a Gemma-3-1B Muon step (training/configs/gemma1b.json:26-34)."""
    return [(layers, 1024, hidden),             # q
            (2 * layers, 256, hidden),          # k, v
            (layers, hidden, 1024),             # o (tall)
            (2 * layers, 6912, hidden),         # gate, up (tall)
            (layers, hidden, 6912)]             # down (wide)


def nanogpt_banks(layers=12, d=768):
    """Bank shapes of the Modded-NanoGPT Muon batch (training/train_nanogpt.py:4881-4888,4918-4919)."""
    return [(4 * layers, d, d), (layers, d, 4 * d), (layers, 4 * d, d)]


def method_table(method):
    return getattr(coefficients, method.upper())
