"""VelvetController — velocity-to-learning-rate translation driven by the
8-bit optimizer's second-moment state (reference packr/velvet.py:22-300).

Same constructor, `warmup_step`, `step` (called after `optimizer.step()`),
`get_stats`, and the same per-parameter arithmetic.  The difference is how
the per-parameter means of `v` are read: the reference dequantises and
averages each parameter with its own `.item()` (one host sync per parameter);
here one packr_state_v_sums launch sums every int8 `v` state on the device
(each code times its block's scale) and a single copy brings all the sums
back.  float32 `v` states (plain AdamW) are averaged with torch on the device
and come back in the same copy.
"""
from __future__ import annotations

import ctypes
from typing import Dict, List, Optional

import torch

from . import _lib


def state_v_sums(items, device) -> torch.Tensor:
    """float64 [len(items)] device tensor: for each (v, v_scale, start, numel,
    block_size) the sum of the int8 codes v[start:start+numel], each times
    v_scale[(start + i) / block_size] when block_size > 0.  One
    packr_state_v_sums launch on the current stream."""
    sums = torch.empty(len(items), dtype=torch.float64, device=device)
    if not items:
        return sums
    lib = _lib.load()
    arr = (_lib.VSumDesc * len(items))()
    for d, (v, vs, start, numel, bs) in zip(arr, items):
        if v.dtype != torch.int8 or not v.is_cuda or not v.is_contiguous():
            raise ValueError("state_v_sums: v must be a contiguous int8 CUDA tensor")
        if start < 0 or start + numel > v.numel():
            raise ValueError("state_v_sums: slice outside v")
        if bs > 0 and (vs is None or vs.dtype != torch.float32 or not vs.is_contiguous()
                       or (start + numel + bs - 1) // bs > vs.numel()):
            raise ValueError("state_v_sums: v_scale must be a contiguous float32 tensor covering the slice")
        d.v = v.data_ptr() + start
        d.v_scale = vs.data_ptr() if bs > 0 else None
        d.numel, d.block_size, d.block_origin = numel, bs, start if bs > 0 else 0
    with torch.cuda.device(device):
        code = lib.packr_state_v_sums(arr, len(items), ctypes.c_void_p(sums.data_ptr()),
                                      ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream))
    _lib.check("packr_state_v_sums", code)
    return sums


def _v_means(states) -> List[float]:
    """Mean of each state's v as reference velvet.py:270-300 defines it, with
    one device->host copy.  `states`: list of (v, v_scale or None)."""
    if not states:
        return []
    dev = states[0][0].device
    int8_idx, items, other = [], [], []
    for i, (v, vs) in enumerate(states):
        if v.dtype == torch.int8:
            if not v.is_cuda:
                raise ValueError("VelvetController: int8 v states are read by the CUDA kernel; this one is on the CPU")
            n = v.numel()
            bs = 0
            if vs is not None:
                nb = vs.numel()
                b = (n + nb - 1) // nb if nb else 0
                if nb and n == nb * b:  # the [blocks, block_size] view exists: scaled mean
                    bs = b
            items.append((v.contiguous().reshape(-1), vs.contiguous().reshape(-1) if bs else None, 0, n, bs))
            int8_idx.append(i)
        else:
            other.append(i)
    parts = []
    if items:
        counts = torch.tensor([max(it[3], 1) for it in items], dtype=torch.float64, device=dev)
        parts.append(state_v_sums(items, dev) / counts)
    if other:
        parts.append(torch.stack([(states[i][0] if states[i][0].dtype == torch.float32 else states[i][0].float())
                                  .mean().to(device=dev, dtype=torch.float64) for i in other]))
    host = torch.cat(parts).cpu().tolist()  # the one device -> host copy
    out = [0.0] * len(states)
    for j, i in enumerate(int8_idx + other):
        out[i] = host[j]
    return out


class VelvetController:
    """Velocity to Learning Rate Translation controller (reference
    packr/velvet.py:22-50 documents the parameters)."""

    def __init__(self, optimizer, beta: float = 0.97, min_multiplier: float = 0.175, max_multiplier: float = 1.0,
                 velocity_scale: float = 10.0, train_samples: Optional[int] = None,
                 total_opt_steps: Optional[int] = None, opt_steps_per_epoch: Optional[int] = None):
        velocity_scale_default = 10.0
        tuning_steps = train_samples
        if tuning_steps is None:
            tuning_steps = opt_steps_per_epoch
        if tuning_steps is None:
            tuning_steps = total_opt_steps
        self._v_ref_beta = 0.97
        self._auto_tuned = False
        self._min_observation_steps = 1
        if tuning_steps is not None and tuning_steps > 0:
            if train_samples is not None:
                scale = min(1.0, (tuning_steps / 32000.0) ** 0.33)
            else:
                scale = min(1.0, (tuning_steps / 1000.0) ** 0.33)
            auto_half_life = max(5, int(25.0 * scale))
            if beta is None:
                beta = 0.5 ** (1.0 / auto_half_life)
                min_multiplier = 0.175 + 0.325 * (1.0 - scale)
                v_ref_half_life = max(3, int(23.0 * scale))
                self._v_ref_beta = 0.5 ** (1.0 / v_ref_half_life)
                self._auto_tuned = True
            if velocity_scale is None:
                velocity_scale = 1.5 + (velocity_scale_default - 1.5) * scale
        if velocity_scale is None:
            velocity_scale = velocity_scale_default
        if beta is None or not 0 < beta < 1:
            raise ValueError(f"beta must be in (0, 1), got {beta}")
        if not 0 <= min_multiplier <= max_multiplier:
            raise ValueError(f"min_multiplier ({min_multiplier}) must be <= max_multiplier ({max_multiplier})")
        self._optimizer = optimizer
        self.beta = beta
        self.min_m = min_multiplier
        self.max_m = max_multiplier
        self.vel_scale = velocity_scale
        self._v_ref: Dict[int, float] = {}
        self._ema_velocity: Dict[int, float] = {}
        self._base_lr: Dict[int, float] = {i: g["lr"] for i, g in enumerate(optimizer.param_groups)}
        self._step_count = 0
        self._stats: Dict[str, list] = {"step": [], "group": [], "v_mean": [], "velocity": [], "multiplier": [],
                                        "lr": []}

    @torch.no_grad()
    def warmup_step(self, global_step: int, warmup_steps: int) -> None:
        """Linear warmup from 10 % to 100 % of each group's base LR
        (reference velvet.py:135-145)."""
        factor = 0.1 + 0.9 * (global_step / max(warmup_steps, 1))
        for group_idx, group in enumerate(self._optimizer.param_groups):
            group["lr"] = self._base_lr[group_idx] * factor

    @torch.no_grad()
    def step(self) -> None:
        """After optimizer.step(): per-group LR from the filtered velocity of
        the v states (reference velvet.py:147-232)."""
        self._step_count += 1
        is_first = self._step_count == 1
        observing = self._step_count <= self._min_observation_steps
        # every tracked parameter's v mean, in one batch
        if hasattr(self._optimizer, "v_means"):  # sharded state: the optimizer combines its shards
            means = self._optimizer.v_means()
            grads = {id(p) for g in self._optimizer.param_groups for p in g["params"] if p.grad is not None}
            means = {pid: m for pid, m in means.items() if pid in grads}
        else:
            means = self._gather_means()
        self._apply(means, is_first, observing)

    def _gather_means(self) -> Dict[int, float]:
        tracked = []
        for group in self._optimizer.param_groups:
            for p in group["params"]:
                if p.grad is None:
                    continue
                state = self._optimizer.state.get(p)
                if state is None or "v" not in state:
                    continue
                tracked.append((p, state["v"], state.get("v_scale")))
        return dict(zip((id(p) for p, _, _ in tracked), _v_means([(v, vs) for _, v, vs in tracked])))

    def _apply(self, means: Dict[int, float], is_first: bool, observing: bool) -> None:
        for group_idx, group in enumerate(self._optimizer.param_groups):
            multipliers: List[float] = []
            for p in group["params"]:
                pid = id(p)
                if pid not in means:
                    continue
                v_mean = means[pid]
                if is_first or pid not in self._v_ref:
                    self._v_ref[pid] = v_mean
                    self._ema_velocity[pid] = 0.0
                    multipliers.append(self.max_m)
                    continue
                v_ref_old = self._v_ref[pid]
                v_ref_new = self._v_ref_beta * v_ref_old + (1.0 - self._v_ref_beta) * v_mean
                self._v_ref[pid] = v_ref_new
                delta = (v_ref_new - v_ref_old) / (1.0 - self._v_ref_beta)
                ema = self.beta * self._ema_velocity[pid] + (1.0 - self.beta) * delta
                self._ema_velocity[pid] = ema
                if observing:
                    multipliers.append(self.max_m)
                    continue
                norm_vel = abs(ema) / (v_ref_new + 1e-12)
                multipliers.append(self.min_m + (self.max_m - self.min_m) * min(1.0, norm_vel * self.vel_scale))
            if multipliers:
                group_m = sum(multipliers) / len(multipliers)
                group["lr"] = self._base_lr[group_idx] * group_m
                sample_id = id(group["params"][0])
                self._stats["step"].append(self._step_count)
                self._stats["group"].append(group_idx)
                self._stats["v_mean"].append(self._v_ref.get(sample_id, 0.0))
                self._stats["velocity"].append(self._ema_velocity.get(sample_id, 0.0))
                self._stats["multiplier"].append(group_m)
                self._stats["lr"].append(group["lr"])

    def get_stats(self) -> dict:
        """Snapshot of the velocity / multiplier statistics (reference
        velvet.py:234-265)."""
        per_group = {}
        for group_idx, group in enumerate(self._optimizer.param_groups):
            gname = group.get("name", f"group_{group_idx}")
            per_group[gname] = {
                "base_lr": self._base_lr.get(group_idx),
                "current_lr": group["lr"],
                "multiplier": group["lr"] / max(self._base_lr.get(group_idx, 1e-12), 1e-12),
            }
        return {
            "step_count": self._step_count, "beta": self.beta, "v_ref_beta": self._v_ref_beta,
            "vel_scale": self.vel_scale, "min_multiplier": self.min_m, "max_multiplier": self.max_m,
            "auto_tuned": self._auto_tuned, "observation_steps": self._min_observation_steps,
            "per_group": per_group,
            "history": {"steps": self._stats["step"][-100:], "multipliers": self._stats["multiplier"][-100:],
                        "velocities": self._stats["velocity"][-100:]},
        }
