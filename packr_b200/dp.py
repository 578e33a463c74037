"""Data-parallel training of PackR layers: gradient reduce-scatter, 8-bit AdamW
on a 1/N shard of the optimizer state per rank, parameter all-gather.

The reference has no distributed code; this is the one parallel strategy the
B200 build adds (one process per GPU, NCCL over NVLink/NVSwitch).

Layout.  The trainable parameters (W_f, lut, bias_f, and any other tensors
passed in) are re-homed into one flat buffer per dtype; each parameter
starts at a multiple of 256 elements, so the 256-element quantisation blocks
of the 8-bit state never straddle two parameters, and the buffer is padded to
a multiple of 256 * world_size so every rank's shard is a whole number of
blocks.  A parameter's `.data` becomes a view of its flat buffer, so the
all-gather writes the updated values in place.

Step (identical collective sequence on every rank):
  1. copy each .grad into the flat gradient buffer (zeros where None).  Each
     parameter carries `_packr_grad_sink = (flat_grad, offset)`: PackRLinear's
     backward writes dW_f straight into that slice while .grad is None, and
     the copy is skipped for a .grad that already is the slice
  2. reduce_scatter_tensor(op=AVG)   -> this rank's averaged gradient shard
  3. packr_adam8_multi over the parameter sub-ranges of the shard (the same
     per-block arithmetic as CUDA8BitAdam, so the result equals the
     single-process step on the averaged gradient)
  4. all_gather_into_tensor           -> every rank holds the new parameters
With world_size 1 the collectives are skipped and the optimizer reads the
flat gradient buffer itself.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.distributed as dist

BLOCK = 256


@dataclass
class _Slot:
    param: torch.Tensor
    offset: int   # element offset in the flat buffer (multiple of BLOCK)
    numel: int


@dataclass
class _Group:
    dtype: torch.dtype
    slots: list = field(default_factory=list)
    total: int = 0
    flat: torch.Tensor | None = None
    grad: torch.Tensor | None = None
    shard_grad: torch.Tensor | None = None
    m: torch.Tensor | None = None
    v: torch.Tensor | None = None
    ms: torch.Tensor | None = None
    vs: torch.Tensor | None = None
    entries: list = field(default_factory=list)  # (p_view, g_view, m, v, ms, vs)


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


class ShardedAdam8:
    """ZeRO-1 data-parallel 8-bit AdamW over `params` (same device).

    adam_fn(entries, lr, b1, b2, eps, bc1, bc2, wd) performs the 8-bit AdamW
    update on a list of (p, g, m, v, m_scale, v_scale) tensors; the default is
    the sm_100a kernel (packr_b200.cuda_adam.adam8_launch).
    """

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, process_group=None,
                 adam_fn=None):
        self.params = [p for p in params if p.requires_grad]
        if not self.params:
            raise ValueError("ShardedAdam8: no trainable parameters")
        self.lr, self.betas, self.eps, self.weight_decay = lr, betas, eps, weight_decay
        self.pg = process_group
        if dist.is_available() and dist.is_initialized():
            self.world = dist.get_world_size(self.pg)
            self.rank = dist.get_rank(self.pg)
        else:
            self.world, self.rank = 1, 0
        if adam_fn is None:
            from .cuda_adam import adam8_launch
            adam_fn = adam8_launch
        self.adam_fn = adam_fn
        self.step_count = 0
        self.device = self.params[0].device
        self.groups: dict[torch.dtype, _Group] = {}
        for p in self.params:
            if p.device != self.device:
                raise ValueError("ShardedAdam8: all parameters must be on one device")
            g = self.groups.setdefault(p.dtype, _Group(p.dtype))
            g.slots.append(_Slot(p, g.total, p.numel()))
            g.total = _round_up(g.total + p.numel(), BLOCK)
        for g in self.groups.values():
            self._build(g)

    # -------------------------------------------------------------- layout
    def _build(self, g: _Group) -> None:
        total = _round_up(max(g.total, 1), BLOCK * self.world)
        g.total = total
        g.flat = torch.zeros(total, dtype=g.dtype, device=self.device)
        g.grad = torch.zeros(total, dtype=g.dtype, device=self.device)
        for s in g.slots:
            g.flat[s.offset:s.offset + s.numel].copy_(s.param.detach().reshape(-1))
            s.param.data = g.flat[s.offset:s.offset + s.numel].view_as(s.param)
            s.param._packr_grad_sink = (g.grad, s.offset)
        shard = total // self.world
        s0 = self.rank * shard
        g.shard_grad = g.grad if self.world == 1 else torch.zeros(shard, dtype=g.dtype, device=self.device)
        g.m = torch.zeros(shard, dtype=torch.int8, device=self.device)
        g.v = torch.zeros(shard, dtype=torch.int8, device=self.device)
        g.ms = torch.ones(shard // BLOCK, dtype=torch.float32, device=self.device)
        g.vs = torch.ones(shard // BLOCK, dtype=torch.float32, device=self.device)
        # parameter sub-ranges inside this rank's shard; both ends of each
        # range are 256-aligned except a parameter's own last element
        for s in g.slots:
            a, b = max(s.offset, s0), min(s.offset + s.numel, s0 + shard)
            if a >= b:
                continue
            la, lb = a - s0, b - s0
            ba, bb = la // BLOCK, (lb + BLOCK - 1) // BLOCK
            g.entries.append((g.flat[a:b], g.shard_grad[la:lb], g.m[la:lb], g.v[la:lb], g.ms[ba:bb], g.vs[ba:bb]))

    @property
    def shard_numel(self) -> int:
        return sum(g.total // self.world for g in self.groups.values())

    # -------------------------------------------------------------- step
    @torch.no_grad()
    def step(self) -> None:
        self.step_count += 1
        b1, b2 = self.betas
        bc1 = 1.0 - b1 ** self.step_count
        bc2 = 1.0 - b2 ** self.step_count
        for dt in sorted(self.groups, key=str):
            g = self.groups[dt]
            for s in g.slots:
                dst = g.grad[s.offset:s.offset + s.numel]
                if s.param.grad is None:
                    dst.zero_()
                elif s.param.grad.data_ptr() != dst.data_ptr():  # not already the slice
                    dst.copy_(s.param.grad.reshape(-1))
            if self.world > 1:
                dist.reduce_scatter_tensor(g.shard_grad, g.grad, op=dist.ReduceOp.AVG, group=self.pg)
            if g.entries:
                self.adam_fn(g.entries, self.lr, b1, b2, self.eps, bc1, bc2, self.weight_decay)
            if self.world > 1:
                shard = g.total // self.world
                mine = g.flat[self.rank * shard:(self.rank + 1) * shard]
                src = mine if self.device.type == "cuda" else mine.clone()
                dist.all_gather_into_tensor(g.flat, src, group=self.pg)

    def zero_grad(self, set_to_none: bool = True) -> None:
        for p in self.params:
            if set_to_none:
                p.grad = None
            elif p.grad is not None:
                p.grad.zero_()

    def state_dict(self) -> dict:
        """This rank's shard of the 8-bit state (int8 m/v, f32 block scales)."""
        return {"step": self.step_count, "world": self.world, "rank": self.rank,
                "groups": {str(dt): {"m": g.m, "v": g.v, "m_scale": g.ms, "v_scale": g.vs}
                           for dt, g in self.groups.items()}}

    def load_state_dict(self, sd: dict) -> None:
        if sd["world"] != self.world or sd["rank"] != self.rank:
            raise ValueError("ShardedAdam8.load_state_dict: saved for a different world size / rank")
        self.step_count = int(sd["step"])
        for dt, g in self.groups.items():
            s = sd["groups"][str(dt)]
            g.m.copy_(s["m"]); g.v.copy_(s["v"]); g.ms.copy_(s["m_scale"]); g.vs.copy_(s["v_scale"])
