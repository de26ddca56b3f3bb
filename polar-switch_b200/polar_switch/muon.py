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
                out_dtype = torch.bfloat16 if group["scale"] == "rms" else params[0].dtype
                stacked.append(muon_directions([p.grad.contiguous() for p in params], moms,
                                               group["momentum"], out_dtype))
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
