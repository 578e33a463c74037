"""VelvetController host logic against the reference controller's recorded
learning rates (float32 v states, read with torch on the CPU exactly as the
reference reads them), constructor auto-tuning and argument checks."""
import numpy as np
import pytest
import torch

from packr_b200 import VelvetController
from velvet_replay import replay


@pytest.mark.parametrize("setting", range(3))
def test_f32_states_match_reference(setting):
    lrs, want, stats, want_stats = replay("f32", setting, torch.device("cpu"))
    np.testing.assert_allclose(lrs, want, rtol=1e-12, atol=0)
    for k in ("step_count", "beta", "v_ref_beta", "vel_scale", "min_multiplier", "max_multiplier", "auto_tuned",
              "observation_steps"):
        assert stats[k] == pytest.approx(want_stats[k], rel=1e-12), k
    np.testing.assert_allclose(stats["history"]["multipliers"], want_stats["history_multipliers"], rtol=1e-12)
    np.testing.assert_allclose(stats["history"]["velocities"], want_stats["history_velocities"], rtol=1e-12, atol=0)


class _Opt:
    def __init__(self, lr=1e-3):
        self.param_groups = [{"params": [torch.nn.Parameter(torch.zeros(4))], "lr": lr}]
        self.state = {}


def test_argument_checks():
    with pytest.raises(ValueError):
        VelvetController(_Opt(), beta=1.0)
    with pytest.raises(ValueError):
        VelvetController(_Opt(), beta=0.0)
    with pytest.raises(ValueError):
        VelvetController(_Opt(), min_multiplier=0.9, max_multiplier=0.5)
    with pytest.raises(ValueError):  # beta=None needs a step count to tune from
        VelvetController(_Opt(), beta=None)


def test_warmup_and_untracked_groups():
    opt = _Opt(lr=2e-3)
    ctl = VelvetController(opt)
    ctl.warmup_step(0, 10)
    assert opt.param_groups[0]["lr"] == pytest.approx(2e-4)
    ctl.warmup_step(5, 10)
    assert opt.param_groups[0]["lr"] == pytest.approx(2e-3 * 0.55)
    ctl.step()  # no grad, no "v" state: the group is left alone
    ctl.step()
    assert opt.param_groups[0]["lr"] == pytest.approx(2e-3 * 0.55)
    assert ctl.get_stats()["step_count"] == 2


def test_default_constructor_steps():
    """Without a step count to tune from, the trend EMA uses 0.97 (the value
    the reference sets whenever beta is given)."""
    opt = _Opt()
    p = opt.param_groups[0]["params"][0]
    p.grad = torch.zeros(4)
    ctl = VelvetController(opt)
    for t in range(4):
        opt.state[p] = {"v": torch.full((4,), 1e-6 * (1 + 0.1 * t))}
        ctl.step()
    assert ctl.get_stats()["v_ref_beta"] == 0.97
    assert 0.175 <= opt.param_groups[0]["lr"] / 1e-3 <= 1.0


def test_int8_state_on_cpu_is_refused():
    opt = _Opt()
    p = opt.param_groups[0]["params"][0]
    p.grad = torch.zeros(4)
    opt.state[p] = {"v": torch.ones(4, dtype=torch.int8), "v_scale": torch.ones(1)}
    with pytest.raises(ValueError):
        VelvetController(opt).step()
