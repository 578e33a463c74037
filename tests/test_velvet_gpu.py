"""VelvetController on int8 second-moment states: the batched sm_100a v-sum
kernel (packr_state_v_sums) against float64 torch sums, the controller
against the reference controller's recorded learning rates, and the
data-parallel optimizer's combined v means."""
import numpy as np
import pytest
import torch

from velvet_replay import replay

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("setting", range(3))
def test_int8_states_match_reference(cuda, setting):
    # the reference averages in float32, the kernel sums in float64: the
    # multipliers agree to 1e-5 (absolute), the lrs to 1e-5 of the base lr
    lrs, want, stats, want_stats = replay("int8", setting, cuda)
    base = np.array([[1e-3, 5e-4, 2e-3]])
    np.testing.assert_allclose(lrs / base, want / base, rtol=0, atol=1e-5)
    np.testing.assert_allclose(stats["history"]["multipliers"], want_stats["history_multipliers"], rtol=0, atol=1e-5)


def test_v_sums_kernel(cuda):
    from packr_b200.velvet import state_v_sums
    g = torch.Generator(device="cpu").manual_seed(0)
    sizes = [0, 1, 255, 256, 1000, 65535, 65536, 65537, 3 * 65536 + 17, 1 << 20]
    items, want = [], []
    for i, n in enumerate(sizes):
        v = torch.randint(0, 128, (n + 40,), generator=g, dtype=torch.int8)
        start = 0 if i % 2 == 0 else 40
        bs = [0, 256, 250, 7][i % 4]
        nb = (start + n + bs - 1) // bs if bs else 0
        vs = torch.rand(max(nb, 1), generator=g) * 1e-6
        codes = v[start:start + n].double()
        if bs:
            idx = (torch.arange(n) + start) // bs
            want.append((codes * vs.double()[idx]).sum().item())
        else:
            want.append(codes.sum().item())
        items.append((v.to(cuda), vs.to(cuda), start, n, bs))
    got = state_v_sums(items, cuda).cpu().numpy()
    np.testing.assert_allclose(got, np.array(want), rtol=1e-12, atol=0)


def test_v_sums_many_parameters(cuda):
    """More descriptors than one launch holds (512 per launch)."""
    from packr_b200.velvet import state_v_sums
    g = torch.Generator(device="cpu").manual_seed(1)
    vs = [torch.randint(0, 128, (int(n),), generator=g, dtype=torch.int8) for n in torch.randint(1, 3000, (1100,), generator=g)]
    items = [(v.to(cuda), None, 0, v.numel(), 0) for v in vs]
    got = state_v_sums(items, cuda).cpu().numpy()
    np.testing.assert_array_equal(got, np.array([v.double().sum().item() for v in vs]))


def test_with_cuda8bit_adam(cuda):
    """The controller drives a real CUDA8BitAdam: the v means it reads are the
    dequantised means of the optimizer's state, and the lr stays in
    [min, max] x base."""
    from packr_b200 import CUDA8BitAdam, PackRLinear, VelvetController
    from packr_b200.velvet import _v_means
    lay = PackRLinear.synthetic(256, 512, device=cuda, seed=5)
    opt = CUDA8BitAdam(list(lay.parameters()), lr=1e-3)
    ctl = VelvetController(opt, total_opt_steps=200)
    g = torch.Generator(device=cuda).manual_seed(0)
    for _ in range(6):
        x = torch.randn(64, 256, generator=g, device=cuda).to(torch.bfloat16)
        opt.zero_grad()
        lay(x).square().mean().backward()
        opt.step()
        ctl.step()
        lr = opt.param_groups[0]["lr"]
        assert 0.175e-3 - 1e-12 <= lr <= 1e-3 + 1e-12
    checked = 0
    for p in lay.parameters():
        st = opt.state.get(p, {})
        if "v" not in st:  # frozen parameters have no state
            continue
        checked += 1
        n, nb = st["v"].numel(), st["v_scale"].numel()
        bs = (n + nb - 1) // nb
        v = st["v"].double()
        want = v.mean().item() if n < nb * bs else (v.view(nb, bs).mean(1) * st["v_scale"].double()).mean().item()
        assert _v_means([(st["v"], st["v_scale"])])[0] == pytest.approx(want, rel=1e-12)
    assert checked >= 2


def test_sharded_adam_v_means(cuda):
    """World size 1: ShardedAdam8.v_means equals the dequantised mean of each
    parameter's slice of the flat state."""
    from packr_b200 import PackRLinear
    from packr_b200.dp import BLOCK, ShardedAdam8
    lays = [PackRLinear.synthetic(256, 300, device=cuda, seed=6), PackRLinear.synthetic(300, 64, device=cuda, seed=7)]
    params = [p for l in lays for p in l.parameters() if p.requires_grad]
    opt = ShardedAdam8(params, lr=1e-3, bucket_bytes=1 << 16)
    g = torch.Generator(device=cuda).manual_seed(0)
    for _ in range(2):
        x = torch.randn(32, 256, generator=g, device=cuda).to(torch.bfloat16)
        opt.zero_grad()
        lays[1](lays[0](x).to(torch.bfloat16)).square().mean().backward()
        opt.step()
    means = opt.v_means()
    for p in params:
        b = opt.bucket_of(p)
        slot = next(s for s in b.slots if s.param is p)
        idx = torch.arange(slot.offset, slot.offset + slot.numel, device=cuda)
        want = (b.v[idx].double() * b.vs[idx // BLOCK].double()).mean().item()
        assert means[id(p)] == pytest.approx(want, rel=1e-12)
