"""The reference's own behavioural tests (tests/test_packr_kernel.py,
tests/test_packr_core.py, tests/test_vram_regression.py,
tests/test_mode_packr_unchanged.py), run against packr_b200 on the GPU with
the same shapes, bounds and VRAM budgets."""
import pytest
import torch

import packr_b200 as packr
from packr_b200 import PackRConfig, compress_model
from packr_b200.kernel import packr_matmul

pytestmark = pytest.mark.gpu
DEV = "cuda"


# ---- tests/test_packr_kernel.py -------------------------------------------
def test_output_shape(cuda):
    x = torch.randn(4, 64, device=DEV)
    W_p = torch.randint(0, 256, (64, 32), dtype=torch.uint8, device=DEV)
    W_f = torch.randn(64, 32, dtype=torch.bfloat16, device=DEV)
    lut = torch.randn(256, device=DEV)
    out = packr_matmul(x, W_p, W_f, lut)
    assert out.shape == (4, 32) and out.dtype == torch.float32


def test_with_bias(cuda):
    x = torch.randn(4, 64, device=DEV)
    W_p = torch.randint(0, 256, (64, 32), dtype=torch.uint8, device=DEV)
    W_f = torch.randn(64, 32, dtype=torch.bfloat16, device=DEV)
    lut = torch.randn(256, device=DEV)
    bias = torch.randn(32, device=DEV)
    out = packr_matmul(x, W_p, W_f, lut, bias=bias)
    ref = packr_matmul(x, W_p, W_f, lut) + bias
    assert out.shape == (4, 32) and torch.allclose(out, ref, atol=1e-5)


def test_matches_nn_linear(cuda):
    K, N, M = 64, 32, 4
    W = torch.randn(K, N, device=DEV)
    q99 = torch.quantile(W.abs().flatten().float(), 0.99).item()
    cb = torch.linspace(-q99, q99, 256, device=DEV)
    W_p = (W.abs().unsqueeze(-1) - cb.abs().unsqueeze(0).unsqueeze(0)).abs().argmin(dim=-1).to(torch.uint8)
    W_f = (W - cb[W_p.long()]).to(torch.bfloat16)
    x = torch.randn(M, K, device=DEV)
    out = packr_matmul(x, W_p, W_f, cb)
    expected = x.float() @ W.float()
    assert ((out - expected).abs().max() / expected.abs().max()) < 0.05


def test_batch_input(cuda):
    for M in [1, 4, 16, 64]:
        x = torch.randn(M, 64, device=DEV)
        W_p = torch.randint(0, 256, (64, 32), dtype=torch.uint8, device=DEV)
        W_f = torch.randn(64, 32, dtype=torch.bfloat16, device=DEV)
        out = packr_matmul(x, W_p, W_f, torch.randn(256, device=DEV))
        assert out.shape == (M, 32)


def test_contiguity_assertion(cuda):
    x = torch.randn(4, 64, device=DEV)
    W_f = torch.randn(64, 32, dtype=torch.bfloat16, device=DEV)
    W_p_big = torch.randint(0, 256, (128, 64), dtype=torch.uint8, device=DEV)
    W_p_nc = W_p_big[:64, :32]
    assert not W_p_nc.is_contiguous()
    with pytest.raises(AssertionError):
        packr_matmul(x, W_p_nc, W_f, torch.randn(256, device=DEV))


# ---- tests/test_packr_core.py ----------------------------------------------
def _model(*dims, bias=False):
    layers = [torch.nn.Linear(a, b, bias=bias) for a, b in zip(dims[:-1], dims[1:])]
    return torch.nn.Sequential(*layers)


def test_forward_shape_and_3d(cuda):
    cfg = PackRConfig(layer_scope="all", gradient_checkpointing=False)
    m = compress_model(_model(64, 32), cfg).to(DEV)
    assert m(torch.randn(8, 64, device=DEV)).shape == (8, 32)
    assert m(torch.randn(2, 4, 64, device=DEV)).shape == (2, 4, 32)
    mb = compress_model(_model(64, 32, bias=True), cfg).to(DEV)
    assert mb(torch.randn(8, 64, device=DEV)).shape == (8, 32)


def test_forward_matches_nn_linear(cuda):
    cfg = PackRConfig(layer_scope="all", gradient_checkpointing=False)
    original = torch.nn.Linear(64, 32, bias=False)
    w = original.weight.data.clone()
    m = compress_model(original, cfg).to(DEV)
    ref = torch.nn.Linear(64, 32, bias=False).to(DEV)
    ref.weight.data.copy_(w.to(DEV))
    x = torch.randn(8, 64, device=DEV)
    a, b = m(x), ref(x)
    assert ((a - b).abs().max() / b.abs().max()) < 0.05


def test_gradient_flow_and_lut_grad(cuda):
    cfg = PackRConfig(layer_scope="all", gradient_checkpointing=False, learnable_lut=True)
    m = compress_model(_model(64, 32), cfg).to(DEV)
    m(torch.randn(8, 64, device=DEV)).sum().backward()
    for name, p in m.named_parameters():
        if p.requires_grad:
            assert p.grad is not None, name
            assert not torch.isnan(p.grad.float()).any(), name
    g = m[0].lut.grad
    assert g is not None and g.shape == (256,) and not torch.isnan(g).any()


def test_gradient_consistency(cuda):
    cfg = PackRConfig(layer_scope="all", gradient_checkpointing=False, learnable_lut=True)
    m = compress_model(_model(64, 32), cfg).to(DEV)
    m(torch.randn(8, 64, device=DEV)).sum().backward()
    g1 = m[0].lut.grad.clone()
    m.zero_grad()
    m(torch.randn(8, 64, device=DEV)).sum().backward()
    assert not torch.allclose(g1, m[0].lut.grad)


def test_two_layer(cuda):
    cfg = PackRConfig(layer_scope="all", gradient_checkpointing=False, learnable_lut=True)
    m = compress_model(_model(64, 32, 16), cfg).to(DEV)
    out = m(torch.randn(8, 64, device=DEV))
    assert out.shape == (8, 16)
    out.sum().backward()
    for name, p in m.named_parameters():
        if p.requires_grad:
            assert p.grad is not None, name


def test_bf16_input_gives_bf16_grad(cuda):
    m = compress_model(_model(64, 32), PackRConfig(layer_scope="all", gradient_checkpointing=False)).to(DEV)
    x = torch.randn(8, 64, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    out = m(x)
    assert out.dtype == torch.float32
    out.sum().backward()
    assert x.grad.dtype == torch.bfloat16


# ---- tests/test_vram_regression.py -----------------------------------------
def _vram_model():
    cfg = PackRConfig(layer_scope="all", gradient_checkpointing=False)
    return compress_model(_model(768, 3072, 768), cfg).cuda()


def test_forward_peak_vram(cuda):
    m = _vram_model()
    x = torch.randn(4, 768, device=DEV)
    for _ in range(3):
        m(x)
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    for _ in range(10):
        m(x)
    torch.cuda.synchronize()
    assert torch.cuda.max_memory_allocated() / 2 ** 20 < 60


def test_full_step_peak_vram(cuda):
    m = _vram_model()
    x = torch.randn(4, 768, device=DEV)
    for _ in range(3):
        m(x).sum().backward()
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    for _ in range(10):
        m(x).sum().backward()
    torch.cuda.synchronize()
    assert torch.cuda.max_memory_allocated() / 2 ** 20 < 120


def test_single_layer_step_vram(cuda):
    cfg = PackRConfig(layer_scope="all", gradient_checkpointing=False)
    m = compress_model(_model(768, 3072), cfg).cuda()
    x = torch.randn(4, 768, device=DEV)
    for _ in range(3):
        m(x).sum().backward()
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    for _ in range(5):
        m(x).sum().backward()
    torch.cuda.synchronize()
    assert torch.cuda.max_memory_allocated() / 2 ** 20 < 80


# ---- tests/test_mode_packr_unchanged.py -------------------------------------
def test_packr_mode_compresses_and_runs(cuda):
    m = compress_model(_model(64, 32), PackRConfig(layer_scope="all"))
    assert "PackRLinear" in type(m[0]).__name__
    m = m.to(DEV)
    assert m(torch.randn(8, 64, device=DEV)).shape == (8, 32)


def test_cuda8bitadam_trains_compressed_model(cuda):
    """End-to-end: a compressed two-layer model's loss goes down under
    CUDA8BitAdam (the reference README's training loop)."""
    torch.manual_seed(0)
    m = compress_model(_model(64, 128, 16, bias=True), PackRConfig(layer_scope="all", gradient_checkpointing=False)).to(DEV)
    opt = packr.CUDA8BitAdam([p for p in m.parameters() if p.requires_grad], lr=1e-2)
    x = torch.randn(256, 64, device=DEV)
    y = torch.randn(256, 16, device=DEV)
    losses = []
    for _ in range(30):
        loss = torch.nn.functional.mse_loss(m(x), y)
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(loss.item())
    assert losses[-1] < 0.9 * losses[0]
