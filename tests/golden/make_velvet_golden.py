"""Generates tests/golden/velvet_golden.npz by running the REFERENCE
package's VelvetController (packr/velvet.py) on a stand-in optimizer whose
second-moment states follow a seeded schedule.

    PACKR_REFERENCE_ROOT=<reference tree> python tests/golden/make_velvet_golden.py

Two scenarios:
  f32   every state's v is float32 (velvet.py:307-308, `v.mean()`); three
        param groups, one parameter with grad None (skipped, velvet.py:171);
        the CPU test replays it.
  int8  int8 codes with float32 per-block v_scale as CUDA8BitAdam keeps them:
        numel a whole number of 256-element blocks (the scaled mean of the
        [blocks, block_size] view, velvet.py:313-320), numel whose
        [blocks, ceil(numel/blocks)] view regroups the codes (1000 -> [4, 250]),
        numel whose view would need padding (the raw-code mean,
        velvet.py:315-317) and a state without v_scale (velvet.py:311-312);
        the GPU test replays it.
Each scenario runs under three constructor settings (fixed beta; beta and
velocity_scale auto-tuned from train_samples; from opt_steps_per_epoch),
with warmup_step calls before the first steps, and records every group's lr
after each call plus get_stats() at the end.
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

if not os.environ.get("PACKR_REFERENCE_ROOT"):
    raise SystemExit("set PACKR_REFERENCE_ROOT to the reference tree (the directory holding packr/)")
REF = Path(os.environ["PACKR_REFERENCE_ROOT"])
sys.dont_write_bytecode = True
sys.path.insert(0, str(REF))

from packr.velvet import VelvetController  # noqa: E402  (the reference controller)

STEPS = 14
WARMUP = 3
SETTINGS = [
    dict(beta=0.97, total_opt_steps=500),
    dict(beta=None, velocity_scale=None, train_samples=6000),
    dict(beta=None, velocity_scale=None, opt_steps_per_epoch=120),
]
# (group, numel, kind) per parameter; kind: f32 | scaled | regrouped | padded | noscale
# (v_scale has ceil(numel/256) blocks; the reference views v as [blocks,
# ceil(numel/blocks)]: 1000 -> [4, 250] "regrouped", 1281 -> [6, 214] would
# need padding so it takes the raw-code mean)
PARAMS = {
    "f32": [(0, 1024, "f32"), (0, 300, "f32"), (1, 4096, "f32"), (1, 77, "f32"), (2, 512, "f32")],
    "int8": [(0, 1024, "scaled"), (0, 1000, "regrouped"), (1, 4096, "scaled"), (1, 300, "noscale"),
             (2, 1281, "padded"), (2, 257, "padded")],
}
NO_GRAD = {"f32": 3, "int8": None}  # index of a parameter whose grad stays None
LRS = [1e-3, 5e-4, 2e-3]


AMPS = [2.0, 0.3, -0.3, 0.05, 0.8, -0.05]  # per parameter: how far v moves (saturated .. nearly flat)


def schedule(kind: str, numel: int, seed: int, amp: float):
    """STEPS states of one parameter: v moves by `amp` (relative) and then
    flattens, with element noise."""
    g = np.random.default_rng(seed)
    out = []
    for t in range(STEPS):
        level = 0.5 * (1.0 + amp * (1.0 - np.exp(-t / 4.0)))
        if kind == "f32":
            v = (level * 1e-6 * g.uniform(0.5, 1.5, numel)).astype(np.float32)
            out.append((v, None))
            continue
        codes = np.clip(np.round(level * 100 * g.uniform(0.3, 1.0, numel)), 0, 127).astype(np.int8)
        nb = (numel + 255) // 256
        scale = (level * 1e-8 * g.uniform(0.5, 2.0, nb)).astype(np.float32)
        out.append((codes, None if kind == "noscale" else scale))
    return out


class StandIn:
    """The attributes VelvetController reads: param_groups and state."""

    def __init__(self, params, no_grad):
        self.param_groups = [{"params": [], "lr": lr, "name": f"g{i}"} for i, lr in enumerate(LRS)]
        self.state = {}
        self.tensors = []
        for i, (grp, numel, kind) in enumerate(params):
            p = torch.nn.Parameter(torch.zeros(numel))
            if i != no_grad:
                p.grad = torch.zeros(numel)
            self.param_groups[grp]["params"].append(p)
            self.tensors.append(p)

    def load(self, states):
        for p, (v, vs) in zip(self.tensors, states):
            st = {"v": torch.from_numpy(v.copy())}
            if vs is not None:
                st["v_scale"] = torch.from_numpy(vs.copy())
            self.state[p] = st


def main():
    out = {}
    meta = {}
    for scen, params in PARAMS.items():
        scheds = [schedule(kind, numel, 1000 * i + 7, AMPS[i]) for i, (_, numel, kind) in enumerate(params)]
        for i in range(len(params)):
            out[f"{scen}/v/{i}"] = np.stack([s[0] for s in scheds[i]])
            if scheds[i][0][1] is not None:
                out[f"{scen}/vs/{i}"] = np.stack([s[1] for s in scheds[i]])
        for k, setting in enumerate(SETTINGS):
            opt = StandIn(params, NO_GRAD[scen])
            ctl = VelvetController(opt, **setting)
            lrs = []
            for t in range(STEPS):
                if t < WARMUP:
                    ctl.warmup_step(t, WARMUP)
                opt.load([scheds[i][t] for i in range(len(params))])
                ctl.step()
                lrs.append([g["lr"] for g in opt.param_groups])
            out[f"{scen}/lr/{k}"] = np.array(lrs, dtype=np.float64)
            st = ctl.get_stats()
            meta[f"{scen}/{k}"] = {key: st[key] for key in ("step_count", "beta", "v_ref_beta", "vel_scale",
                                                          "min_multiplier", "max_multiplier", "auto_tuned",
                                                          "observation_steps")}
            meta[f"{scen}/{k}"]["history_multipliers"] = st["history"]["multipliers"]
            meta[f"{scen}/{k}"]["history_velocities"] = st["history"]["velocities"]
    out["meta"] = np.frombuffer(json.dumps({"settings": SETTINGS, "params": PARAMS, "no_grad": NO_GRAD, "lrs": LRS,
                                            "steps": STEPS, "warmup": WARMUP, "stats": meta}).encode(),
                                dtype=np.uint8)
    path = Path(__file__).with_name("velvet_golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({path.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
