"""Replays a scenario of tests/golden/velvet_golden.npz (made by the
reference's VelvetController) through packr_b200.VelvetController."""
import json
from pathlib import Path

import numpy as np
import torch

GOLD = np.load(Path(__file__).resolve().parent / "golden" / "velvet_golden.npz")
META = json.loads(bytes(GOLD["meta"]).decode())


class StandIn:
    """The attributes VelvetController reads: param_groups and state."""

    def __init__(self, scen, device):
        self.param_groups = [{"params": [], "lr": lr, "name": f"g{i}"} for i, lr in enumerate(META["lrs"])]
        self.state = {}
        self.tensors = []
        self.device = device
        for i, (grp, numel, _) in enumerate(META["params"][scen]):
            p = torch.nn.Parameter(torch.zeros(numel, device=device))
            if i != META["no_grad"][scen]:
                p.grad = torch.zeros(numel, device=device)
            self.param_groups[grp]["params"].append(p)
            self.tensors.append(p)
        self.scen = scen

    def load(self, t):
        for i, p in enumerate(self.tensors):
            st = {"v": torch.from_numpy(GOLD[f"{self.scen}/v/{i}"][t].copy()).to(self.device)}
            if f"{self.scen}/vs/{i}" in GOLD.files:
                st["v_scale"] = torch.from_numpy(GOLD[f"{self.scen}/vs/{i}"][t].copy()).to(self.device)
            self.state[p] = st


def replay(scen, setting_idx, device):
    from packr_b200 import VelvetController
    opt = StandIn(scen, device)
    ctl = VelvetController(opt, **META["settings"][setting_idx])
    lrs = []
    for t in range(META["steps"]):
        if t < META["warmup"]:
            ctl.warmup_step(t, META["warmup"])
        opt.load(t)
        ctl.step()
        lrs.append([g["lr"] for g in opt.param_groups])
    return np.array(lrs), GOLD[f"{scen}/lr/{setting_idx}"], ctl.get_stats(), META["stats"][f"{scen}/{setting_idx}"]
