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
  * `ShardedOrthogonalizer` runs the local slices as one grouped circuit whose
    FP16 results land directly in a packed send buffer (the circuit rounds to
    FP16, so FP16 is lossless), then one NCCL all_gather_into_tensor gives
    every rank all updates. With one rank nothing is communicated.
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


class ShardedOrthogonalizer:
    """Orthogonalize banks of matrices across the ranks of a process group.

    Every rank passes the same list of banks (CUDA tensors (L_g, rows_g,
    cols_g), e.g. momentum buffers after gradient averaging); each rank
    orthogonalizes its slice of every bank and the FP16 results are
    all-gathered. ``__call__`` returns the gathered buffer; ``bank_updates``
    gives, per bank, the (start, view) slices of the result.
    """

    def __init__(self, bank_shapes, method="PS2_55", epsilon=1e-7, group=None, device=None,
                 world_size=None, rank=None, grouped_fn=None):
        """``grouped_fn(inputs, outs)`` replaces the B200 grouped circuit (used by
        the CPU tests of the sharding logic); by default the circuit runs on
        the GPU."""
        self.group = group
        if world_size is None:
            world_size = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        if rank is None:
            rank = dist.get_rank(group) if world_size > 1 else 0
        self.world_size, self.rank = world_size, rank
        self.polar = make_polynomial_orthogonalizer(method, epsilon=epsilon)
        self.grouped_fn = grouped_fn or (lambda inputs, outs: self.polar.grouped(inputs, outs=outs))
        table = self.polar.table
        self.flops_fn = lambda r, c: circuit_flops(table, r, c)
        self.bank_shapes = [tuple(int(v) for v in s) for s in bank_shapes]
        self.slices = plan_shards(self.bank_shapes, world_size, self.flops_fn)
        self.seg_elems = []
        for rank_slices in self.slices:
            self.seg_elems.append(sum(c * r * k for (_, c), (_, r, k) in zip(rank_slices, self.bank_shapes)))
        # Pad every rank's segment to a multiple of 128 elements (256 B) so the
        # per-problem outputs stay 16-byte aligned.
        self.seg = max(-(-e // 128) * 128 for e in self.seg_elems) if self.seg_elems else 0
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = torch.device(device)
        # In-place all-gather: this rank's segment of the receive buffer is the
        # send buffer, so the circuit writes its results where they end up.
        self.recv = torch.empty(world_size * max(self.seg, 1), device=self.device, dtype=torch.float16)
        self.send = self.recv[rank * self.seg:(rank + 1) * self.seg]
        self.flops_total = sum(L * self.flops_fn(r, c) for L, r, c in self.bank_shapes)
        self.flops_per_rank = plan_loads(self.bank_shapes, self.slices, self.flops_fn)

    def _segment_views(self, buf, rank):
        """Views of one rank's packed segment, one per non-empty bank slice."""
        views, off = [], 0
        for g, ((start, count), (_, rows, cols)) in enumerate(zip(self.slices[rank], self.bank_shapes)):
            if count:
                n = count * rows * cols
                views.append((g, start, buf[off:off + n].view(count, rows, cols)))
                off += n
        return views

    def compute_local(self, banks):
        """Orthogonalize this rank's slices into the packed send buffer (no communication)."""
        if len(banks) != len(self.bank_shapes):
            raise ValueError("expected one tensor per bank")
        for X, shape in zip(banks, self.bank_shapes):
            if tuple(X.shape) != shape:
                raise ValueError(f"bank shape {tuple(X.shape)} does not match the plan {shape}")
        inputs, outputs = [], []
        for g, start, view in self._segment_views(self.send, self.rank):
            inputs.append(banks[g][start:start + view.shape[0]])
            outputs.append(view)
        if inputs:
            self.grouped_fn(inputs, outputs)
        return self.send

    def __call__(self, banks):
        """Orthogonalize all banks across the group; returns the gathered FP16 buffer."""
        self.compute_local(banks)
        if self.world_size > 1:
            dist.all_gather_into_tensor(self.recv, self.send, group=self.group)
        return self.recv

    def bank_updates(self):
        """Per bank, the list of (start, FP16 view) slices of the gathered result."""
        out = [[] for _ in self.bank_shapes]
        for r in range(self.world_size):
            seg = self.recv[r * self.seg:(r + 1) * self.seg]
            for g, start, view in self._segment_views(seg, r):
                out[g].append((start, view))
        return out

    def gathered_banks(self):
        """The full update of every bank as one FP16 tensor each (copies)."""
        res = []
        for g, parts in enumerate(self.bank_updates()):
            parts.sort(key=lambda p: p[0])
            res.append(torch.cat([v for _, v in parts]) if parts else None)
        return res


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
