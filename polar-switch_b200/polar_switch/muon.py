"""Muon on B200: the reference optimizer (training/muon.py) with its per-step
work around the orthogonalizer moved onto the library.

Same groups, arguments, update rule and rounding as the reference's `Muon`
(training/muon.py:31-86): Nesterov momentum, BF16 directions for the "rms"
scale, the polar approximation of every same-shape bucket, then decoupled
weight decay and the scaled update. Two things differ in how it runs:

  * the momentum update, the Nesterov direction, the stacking of a bucket and
    the cast are one kernel per bucket (ps_muon_direction) instead of four
    elementwise passes per matrix;
  * when the orthogonalizer has ``grouped`` (every orthogonalizer of this
    package except GNS), all buckets of a parameter group are orthogonalized
    in one grouped call;
  * the decoupled weight decay and the scaled update are one kernel per
    bucket (ps_muon_update) instead of three elementwise passes per matrix.

`parameter_groups` is the reference's grouping (training/muon.py:14-28).

`ShardedMuon` is the same update run across ranks the way the reference's
NanoGPT optimizer shards its parameter banks (train_nanogpt.py:3983-4037):
gradients averaged and scattered in chunks of whole matrices, momentum kept
only for the local chunk, one grouped orthogonalization of all local chunks,
and the updated chunks gathered back into every rank's banks.
"""

import ctypes
import math

import torch

from . import _native as nat


def parameter_groups(model):
    """Hidden matrix weights by layer role, and the parameters for AdamW
    (embeddings, the output head and non-matrices), as the reference does."""
    matrices, scalars = {}, []
    for name, parameter in model.named_parameters():
        if parameter.ndim != 2 or any(s in name for s in ("embed_tokens", "lm_head")):
            scalars.append(parameter)
        else:
            matrices.setdefault(name.split(".")[-2], []).append(parameter)
    return [{"params": params, "role": role} for role, params in sorted(matrices.items())], scalars


def muon_directions(grads, moms, momentum, out_dtype, nesterov=True):
    """Update the momentum buffers in place and return the stacked directions
    (len(grads), *shape) in `out_dtype` (one kernel per bucket)."""
    g0 = grads[0]
    if not g0.is_cuda:
        raise NotImplementedError("muon_directions: polar_switch_b200 runs on CUDA tensors only")
    for t in list(grads) + list(moms):
        if t.shape != g0.shape or t.dtype != g0.dtype or not t.is_contiguous() or t.device != g0.device:
            raise ValueError("muon_directions: a bucket needs contiguous tensors of one shape, dtype and device")
    out = torch.empty((len(grads), *g0.shape), device=g0.device, dtype=out_dtype)
    gp = (ctypes.c_void_p * len(grads))(*[t.data_ptr() for t in grads])
    mp = (ctypes.c_void_p * len(moms))(*[t.data_ptr() for t in moms])
    with torch.cuda.device(g0.device):
        nat.check("ps_muon_direction", nat.load().ps_muon_direction(
            gp, mp, len(grads), g0.numel(), nat.DTYPE_CODES[g0.dtype], float(momentum), 1 if nesterov else 0,
            nat.ptr(out), nat.DTYPE_CODES[out_dtype], nat.stream_ptr(g0.device)))
    return out


def fused_direction_ok(params, grads, moms):
    """Whether ps_muon_direction can take this bucket: every momentum buffer
    contiguous and every gradient and buffer in the parameters' dtype (a
    non-contiguous gradient is copied to a contiguous one first). Otherwise
    the bucket takes the reference's elementwise sequence: a parameter that is
    a transposed view has a momentum buffer with its strides (zeros_like keeps
    them), and FP32 gradients on BF16 weights promote the direction to FP32."""
    dtype = params[0].dtype
    return (dtype in (torch.float32, torch.bfloat16, torch.float16)
            and all(g.dtype == dtype for g in grads)
            and all(m.dtype == dtype and m.is_contiguous() for m in moms))


def reference_directions(grads, moms, momentum, rms):
    """The reference's direction step for one bucket (training/muon.py:66-76),
    in torch: buf <- momentum * buf + g; d = g + momentum * buf; the stacked
    directions cast to BF16 for the "rms" scale, else kept in the promoted dtype."""
    directions = []
    for g, buf in zip(grads, moms):
        buf.mul_(momentum).add_(g)
        directions.append(g.add(buf, alpha=momentum))
    update = torch.stack(directions)
    return update.bfloat16() if rms else update


def muon_update(params, update, decay, alpha):
    """p <- p * decay + alpha * u for each matrix p and its row u of the stacked
    `update`, rounded like torch's p.mul_(decay); p.add_(u.to(p.dtype), alpha)."""
    p0 = params[0]
    if not p0.is_cuda:
        raise NotImplementedError("muon_update: polar_switch_b200 runs on CUDA tensors only")
    for p in params:
        if p.shape != p0.shape or p.dtype != p0.dtype or not p.is_contiguous() or p.device != p0.device:
            raise ValueError("muon_update: a bucket needs contiguous tensors of one shape, dtype and device")
    if update.shape != (len(params), *p0.shape) or not update.is_contiguous() or update.device != p0.device:
        raise ValueError("muon_update: the update must be the stacked (count, *shape) result")
    pp = (ctypes.c_void_p * len(params))(*[p.data_ptr() for p in params])
    with torch.cuda.device(p0.device):
        nat.check("ps_muon_update", nat.load().ps_muon_update(
            pp, len(params), p0.numel(), nat.DTYPE_CODES[p0.dtype], nat.ptr(update),
            nat.DTYPE_CODES[update.dtype], float(decay), float(alpha), nat.stream_ptr(p0.device)))


class Muon(torch.optim.Optimizer):
    """Nesterov Muon with a polar approximation from make_polynomial_orthogonalizer
    (arguments as training/muon.py:Muon)."""

    def __init__(self, groups, orthogonalize, lr, momentum=0.95, weight_decay=0.0, scale="rms",
                 norm_log=None, parameter_names=None):
        super().__init__(groups, dict(lr=lr, momentum=momentum, weight_decay=weight_decay, scale=scale))
        self.orthogonalize = orthogonalize
        self.norm_log = norm_log
        self.parameter_names = parameter_names or {}

    @torch.no_grad()
    def step(self):
        """Update parameters from their gradients using momentum and the polar approximation."""
        for group in self.param_groups:
            buckets = {}
            for p in group["params"]:
                if p.grad is not None:
                    buckets.setdefault((tuple(p.shape), p.dtype, p.device), []).append(p)
            if not buckets:
                continue
            stacked, members = [], []
            for params in buckets.values():
                moms = []
                for p in params:
                    state = self.state[p]
                    if "momentum_buffer" not in state:
                        state["momentum_buffer"] = torch.zeros_like(p)
                    moms.append(state["momentum_buffer"])
                # BF16 directions for the "rms" scale, as the reference passes them.
                rms = group["scale"] == "rms"
                grads = [p.grad for p in params]
                if fused_direction_ok(params, grads, moms):
                    out_dtype = torch.bfloat16 if rms else params[0].dtype
                    stacked.append(muon_directions([g.contiguous() for g in grads], moms,
                                                   group["momentum"], out_dtype))
                else:
                    stacked.append(reference_directions(grads, moms, group["momentum"], rms))
                members.append(params)
            grouped = getattr(self.orthogonalize, "grouped", None)
            updates = grouped(stacked) if grouped is not None else [self.orthogonalize(u) for u in stacked]
            for params, update in zip(members, updates):
                if self.norm_log is not None:
                    self.norm_log.record(group["role"], update,
                                         execution=self.orthogonalize.last_execution,
                                         matrix_names=[self.parameter_names.get(id(p)) for p in params])
                rows, cols = params[0].shape
                factor = (0.2 * math.sqrt(max(rows, cols)) if group["scale"] == "rms"
                          else math.sqrt(rows / cols))
                if all(p.is_contiguous() for p in params) and update.is_contiguous():
                    muon_update(params, update, 1 - group["lr"] * group["weight_decay"],
                                -group["lr"] * factor)
                else:
                    for p, u in zip(params, update.unbind()):
                        p.mul_(1 - group["lr"] * group["weight_decay"])
                        p.add_(u.to(p.dtype), alpha=-group["lr"] * factor)


def padded_count(count, world_size):
    """Matrices a bank holds so that every rank owns the same number: count
    rounded up to a multiple of world_size, the extra matrices zero (the
    reference's next_multiple_of_n, train_nanogpt.py:4880-4888)."""
    return -(-int(count) // int(world_size)) * int(world_size)


def check_banks(banks, world_size):
    """Raise ValueError unless every bank is a contiguous (count, rows, cols)
    tensor whose count splits evenly over world_size ranks."""
    for bank in banks:
        if bank.ndim != 3 or not bank.is_contiguous():
            raise ValueError("ShardedMuon: each parameter must be a contiguous (count, rows, cols) bank")
        if bank.shape[0] % world_size:
            raise ValueError(f"ShardedMuon: a bank of {bank.shape[0]} matrices does not split over "
                             f"{world_size} ranks; pad it to padded_count()")


class ShardedMuon(torch.optim.Optimizer):
    """Nesterov Muon over parameter banks sharded across ranks.

    Each parameter is a bank of same-shape matrices, shape (count, rows, cols)
    with count a multiple of the world size (`padded_count`; padding matrices
    are zero and stay zero). Per step, as the reference's NanoGPT optimizer
    (train_nanogpt.py:3983-4037, `_launch_reduce` / `_launch_gather`):

      1. every bank's gradient is averaged over ranks and scattered, rank r
         receiving matrices [r * chunk, (r + 1) * chunk) (reduce_scatter_tensor,
         AVG; all banks' scatters are in flight before the first is used);
      2. the momentum of the local chunk is updated and its Nesterov direction
         formed (ps_muon_direction, one kernel per bank; BF16 directions for
         the "rms" scale);
      3. the local chunks of all banks are orthogonalized in one grouped call;
      4. the local slice of every bank gets the decoupled weight decay and the
         scaled update -- by default inside the last apply of its circuit
         (ps_circuit_grouped_update: the update never exists in memory), else
         with ps_muon_update -- and all_gather_into_tensor writes every rank's
         slice into every rank's bank.

    With a `norm_log` (polar_switch.diagnostics.NormLog) every local chunk's
    orthogonalized update is recorded before it is applied, labelled with the
    bank's `label` attribute (else its group's "role") and starting at matrix
    rank * chunk, as train_nanogpt.py:4276-4278 records it.

    The update rule and its rounding are those of `Muon` (training/muon.py:
    54-86), so at world size 1 the two optimizers give the same bits. Runs on
    CUDA banks (NCCL between ranks); with no process group it is world size 1.
    The collectives pair up bank by bank in parameter order, so every rank
    must hold gradients for the same banks, as data-parallel training gives
    (a bank with no gradient on any rank is skipped by all). Checking this
    at run time would cost a host synchronisation per step, so it is not
    checked.
    """

    def __init__(self, banks, orthogonalize, lr, momentum=0.95, weight_decay=0.0, scale="rms",
                 group=None, norm_log=None, fuse_update=True):
        banks = list(banks)
        super().__init__(banks, dict(lr=lr, momentum=momentum, weight_decay=weight_decay, scale=scale))
        self.orthogonalize = orthogonalize
        self.group = group
        self.norm_log = norm_log
        self.fuse_update = fuse_update
        if torch.distributed.is_available() and torch.distributed.is_initialized():
            self.world_size = torch.distributed.get_world_size(group)
            self.rank = torch.distributed.get_rank(group)
        else:
            self.world_size, self.rank = 1, 0
        check_banks([b for g in self.param_groups for b in g["params"]], self.world_size)

    def _chunk(self, bank):
        n = bank.shape[0] // self.world_size
        return n, bank[self.rank * n:(self.rank + 1) * n]

    def _directions(self, grad_chunk, mom_chunk, momentum, out_dtype):
        return muon_directions(list(grad_chunk.unbind(0)), list(mom_chunk.unbind(0)), momentum, out_dtype)

    def _update(self, param_chunk, update, decay, alpha):
        muon_update(list(param_chunk.unbind(0)), update, decay, alpha)

    def _fusable(self, grouped, entries):
        """Whether the update can be folded into the orthogonalization: this
        package's grouped orthogonalizer, no update log (it needs the update
        tensor), the library's own update step, and banks the update-fused
        circuit takes (CUDA, FP32/BF16/FP16, rows and columns multiples of 8;
        the CTA-pair kernel, the default, is checked by the library)."""
        if (not self.fuse_update or grouped is None or self.norm_log is not None
                or type(self)._update is not ShardedMuon._update):
            return False
        return all(bank.is_cuda and bank.dtype in (torch.float32, torch.bfloat16, torch.float16)
                   and bank.shape[-1] % 8 == 0 and bank.shape[-2] % 8 == 0 for _, bank, _, _ in entries)

    @torch.no_grad()
    def step(self):
        """One optimizer step from the banks' (unreduced, per-rank) gradients."""
        dist = torch.distributed
        W = self.world_size
        entries = []  # (group, bank, local gradient chunk, pending scatter)
        for g in self.param_groups:
            for bank in g["params"]:
                if bank.grad is None:
                    continue
                grad = bank.grad.contiguous()
                n, _ = self._chunk(bank)
                if W == 1:
                    entries.append((g, bank, grad, None))
                    continue
                local = torch.empty((n, *grad.shape[1:]), device=grad.device, dtype=grad.dtype)
                work = dist.reduce_scatter_tensor(local, grad, op=dist.ReduceOp.AVG, group=self.group,
                                                  async_op=True)
                entries.append((g, bank, local, work))
        if not entries:
            return
        directions = []
        for g, bank, local, work in entries:
            if work is not None:
                work.wait()
            state = self.state[bank]
            if "momentum_chunk" not in state:
                state["momentum_chunk"] = torch.zeros_like(local)
            out_dtype = torch.bfloat16 if g["scale"] == "rms" else bank.dtype
            directions.append(self._directions(local, state["momentum_chunk"], g["momentum"], out_dtype))
        grouped = getattr(self.orthogonalize, "grouped", None)
        if self._fusable(grouped, entries):
            # Step 4 folded into the circuits' last applies: each local slice
            # receives its update inside the kernel that computes it.
            targets = []
            for g, bank, _, _ in entries:
                rows, cols = bank.shape[-2:]
                factor = (0.2 * math.sqrt(max(rows, cols)) if g["scale"] == "rms"
                          else math.sqrt(rows / cols))
                targets.append((self._chunk(bank)[1], 1 - g["lr"] * g["weight_decay"], -g["lr"] * factor))
            grouped(directions, updates=targets)
            if W > 1:
                works = [dist.all_gather_into_tensor(bank.data, self._chunk(bank)[1], group=self.group,
                                                     async_op=True) for _, bank, _, _ in entries]
                for work in works:
                    work.wait()
            return
        updates = grouped(directions) if grouped is not None else [self.orthogonalize(d) for d in directions]
        gathers = []
        for i, ((g, bank, _, _), update) in enumerate(zip(entries, updates)):
            if self.norm_log is not None:
                label = getattr(bank, "label", None) or g.get("role") or f"bank{i}"
                self.norm_log.record(label, update, self.rank * (bank.shape[0] // W),
                                     execution=getattr(self.orthogonalize, "last_execution", None))
            rows, cols = bank.shape[-2:]
            factor = (0.2 * math.sqrt(max(rows, cols)) if g["scale"] == "rms" else math.sqrt(rows / cols))
            _, mine = self._chunk(bank)
            self._update(mine, update.contiguous(), 1 - g["lr"] * g["weight_decay"], -g["lr"] * factor)
            if W > 1:
                gathers.append(dist.all_gather_into_tensor(bank.data, mine, group=self.group, async_op=True))
        for work in gathers:
            work.wait()
