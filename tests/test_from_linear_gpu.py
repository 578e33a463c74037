"""PackRLinear.from_linear on the GPU (packr_abs_order_stats +
packr_from_linear_encode): the order statistics against a full sort, the
quantile against torch.quantile, the compressed layer against the reference's
own outputs (golden fixtures) and against the reference's torch operation
sequence run on the weight's own device (f32, bf16 and f16 weights, on the
GPU or in host memory), and a weight above torch.quantile's 2^24-element
limit."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import reference_port
from packr_b200 import PackRLinear
from packr_b200 import kernel

pytestmark = pytest.mark.gpu

GOLD = np.load(Path(__file__).resolve().parent / "golden" / "packr_linear_golden.npz")


def bits(t):
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n", [1, 2, 7, 1000, 4099, 65536 + 3, 1 << 20])
def test_order_stats_match_sort(cuda, dtype, n):
    g = torch.Generator(device="cpu").manual_seed(n)
    w = (torch.randn(n + 1, generator=g) * 0.02).to(dtype)
    w[: n // 3] = w[n // 3: 2 * (n // 3)]          # duplicates
    w = w[1:].to(cuda)                             # an offset view (unaligned for the vector loads)
    srt = torch.sort(w.abs().float()).values
    for lo in sorted({0, n // 2, max(n - 2, 0), int(0.99 * (n - 1))}):
        for hi in (lo, lo + 1):
            if hi >= n:
                continue
            got = kernel.abs_order_stats(w, lo, hi).cpu()
            assert got[0].item() == srt[lo].item() and got[1].item() == srt[hi].item(), (lo, hi)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n", [3, 1000, 3 * 1024 * 1024 + 5])
def test_quantile_matches_torch(cuda, dtype, n):
    g = torch.Generator(device="cpu").manual_seed(7)
    w = (torch.randn(n, generator=g) * 0.05).to(dtype).to(cuda)
    want = torch.quantile(w.abs().float(), 0.99)
    got = kernel.quantile_abs(w, 0.99)
    assert got.item() == want.item()


@pytest.mark.parametrize("name", ["fl_small", "fl_wide"])
def test_from_linear_matches_reference_golden(cuda, name):
    w = torch.from_numpy(GOLD[f"{name}/weight"].copy())
    has_b = f"{name}/bias" in GOLD.files
    lin = torch.nn.Linear(w.shape[1], w.shape[0], bias=has_b)
    with torch.no_grad():
        lin.weight.copy_(w)
        if has_b:
            lin.bias.copy_(torch.from_numpy(GOLD[f"{name}/bias"].copy()))
    pk = PackRLinear.from_linear(lin.to(cuda))
    assert np.array_equal(bits(pk.W_p), GOLD[f"{name}/W_p"])
    assert np.array_equal(bits(pk.W_f), GOLD[f"{name}/W_f"])
    assert np.array_equal(bits(pk.lut), GOLD[f"{name}/lut"])
    if has_b:
        assert np.array_equal(bits(pk.bias_f), GOLD[f"{name}/bias_f"])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(77, 300), (513, 1000), (64, 64), (1, 5)])
def test_from_linear_matches_torch_sequence(cuda, dtype, shape):
    out_f, in_f = shape
    torch.manual_seed(out_f * 7 + in_f)
    lin = torch.nn.Linear(in_f, out_f, bias=True).to(device=cuda, dtype=dtype)
    with torch.no_grad():
        lin.weight.mul_(3.0)
        lin.weight[0, 0] = 0.0
    fast = PackRLinear.from_linear(lin)
    ref = reference_port.from_linear(lin.weight, lin.bias)
    assert torch.equal(fast.W_p, ref["W_p"])
    assert np.array_equal(bits(fast.W_f), bits(ref["W_f"]))
    assert np.array_equal(bits(fast.lut), bits(ref["lut"]))
    assert torch.equal(fast.bias_f, ref["bias_f"])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_from_linear_of_host_weight(cuda, dtype):
    """A Linear held in host memory is compressed by the same kernels on the
    current GPU; the new layer's tensors come back to the host and equal the
    reference's sequence on the host (for bf16 torch's CPU kernel rounds
    W * scale differently from its CUDA kernel, and the host's rounding is
    the one reproduced)."""
    torch.manual_seed(11)
    lin = torch.nn.Linear(300, 130, bias=True).to(dtype)
    pk = PackRLinear.from_linear(lin)
    assert all(t.device.type == "cpu" for t in (pk.W_p, pk.W_f, pk.lut, pk.bias_f))
    ref = reference_port.from_linear(lin.weight, lin.bias)
    assert torch.equal(pk.W_p, ref["W_p"])
    assert np.array_equal(bits(pk.W_f), bits(ref["W_f"]))
    assert np.array_equal(bits(pk.lut), bits(ref["lut"]))
    assert torch.equal(pk.bias_f, ref["bias_f"])


@pytest.mark.parametrize("home", ["cuda", "cpu"])
def test_from_linear_of_f16_weight(cuda, home):
    """An f16 weight (on the GPU or the host) equals the reference's f16
    sequence on the same device: W * scale rounded to f16 with the
    multiplier torch uses there, the clamp at f16(1.6)."""
    torch.manual_seed(12)
    lin = torch.nn.Linear(256, 192, bias=True).to(dtype=torch.float16)
    with torch.no_grad():
        lin.weight.mul_(3.0)
    lin = lin.to(home)
    pk = PackRLinear.from_linear(lin)
    ref = reference_port.from_linear(lin.weight, lin.bias)
    assert pk.W_p.device.type == home
    assert torch.equal(pk.W_p, ref["W_p"])
    assert np.array_equal(bits(pk.W_f), bits(ref["W_f"]))
    assert np.array_equal(bits(pk.lut), bits(ref["lut"]))
    assert torch.equal(pk.bias_f, ref["bias_f"])


def test_from_linear_beyond_quantile_limit(cuda):
    """4608 x 4096 bf16 (18.9 M > 2^24 weights): the reference's
    torch.quantile refuses it; here the layer reconstructs W."""
    torch.manual_seed(0)
    lin = torch.nn.Linear(4096, 4608, bias=False).to(device=cuda, dtype=torch.bfloat16)
    pk = PackRLinear.from_linear(lin)
    W = lin.weight.detach().t().float()
    rec = pk.lut[pk.W_p.long()] + pk.W_f.float()
    assert (rec - W).abs().max().item() <= 2 ** -8 * W.abs().max().item()
    # the quantile equals the exact order statistics of a full sort
    n = W.numel()
    a = torch.sort(W.abs().reshape(-1)).values
    pos = torch.tensor(0.99, dtype=torch.float32) * (n - 1)
    lo, hi = int(torch.floor(pos)), int(torch.ceil(pos))
    want = torch.lerp(a[lo], a[hi], (pos - lo).to(cuda))
    assert kernel.quantile_abs(lin.weight, 0.99).item() == want.item()
