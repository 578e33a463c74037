"""Host-side logic that needs no GPU: model surgery, the oracle's from_linear
restatement against the reference's own compression (golden), config, API
surface and the loud failure of the GPU-only ops on CPU tensors."""
from pathlib import Path

import numpy as np
import pytest
import torch

import packr_b200 as packr
from packr_b200 import PackRConfig, PackRLinear, compress_model
from packr_b200.layer import _build_codebook
from oracle import reference_port

GOLD = np.load(Path(__file__).resolve().parent / "golden" / "packr_linear_golden.npz")


def bits(t):
    t = t.detach().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


@pytest.mark.parametrize("name", ["fl_small", "fl_wide"])
def test_oracle_from_linear_matches_reference(name):
    """The oracle's restatement of the reference's from_linear (the checker of
    the GPU path) reproduces the reference's own outputs bit for bit."""
    w = torch.from_numpy(GOLD[f"{name}/weight"].copy())
    has_b = f"{name}/bias" in GOLD.files
    b = torch.from_numpy(GOLD[f"{name}/bias"].copy()) if has_b else None
    r = reference_port.from_linear(w, b)
    assert np.array_equal(bits(r["W_p"]), GOLD[f"{name}/W_p"])
    assert np.array_equal(bits(r["lut"]), GOLD[f"{name}/lut"])
    assert np.array_equal(bits(r["W_f"]), GOLD[f"{name}/W_f"])
    if has_b:
        assert np.array_equal(bits(r["bias_f"]), GOLD[f"{name}/bias_f"])


def test_from_linear_needs_a_gpu():
    """No CPU path: without a CUDA device from_linear refuses loudly."""
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    with pytest.raises(RuntimeError):
        PackRLinear.from_linear(torch.nn.Linear(8, 4))


def test_codebook_definition():
    cb = _build_codebook()
    assert torch.equal(cb, reference_port.codebook())
    for i in (0, 15, 16, 255, 0x5A):
        g, s = i & 15, (i >> 4) & 15
        assert cb[i].item() == np.float32(((g - 7.5) / 7.5) * ((s + 1.0) / 10.0))


def test_quantile_above_torch_limit_matches_order_statistics():
    g = torch.Generator().manual_seed(0)
    w = torch.randn((1 << 24) + 5, generator=g)
    q = reference_port.quantile_abs(w, 0.99).item()
    a = np.sort(np.abs(w.numpy()).astype(np.float64))
    pos = 0.99 * (a.size - 1)
    lo = int(np.floor(pos))
    want = a[lo] + (a[lo + 1] - a[lo]) * (pos - lo)
    assert abs(q - want) <= 1e-6 * want


def test_compress_model_scopes(monkeypatch):
    """Which layers compress_model replaces (the name-scope rules); the
    conversion itself runs on a GPU and is stubbed here."""
    monkeypatch.setattr(PackRLinear, "from_linear",
                        classmethod(lambda cls, lin: cls(lin.in_features, lin.out_features, lin.bias is not None)))

    class Block(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.attention = torch.nn.Module()
            self.attention.query = torch.nn.Linear(16, 16)
            self.attention.output = torch.nn.Module()
            self.attention.output.dense = torch.nn.Linear(16, 16)
            self.intermediate = torch.nn.Module()
            self.intermediate.dense = torch.nn.Linear(16, 64)
            self.output = torch.nn.Module()
            self.output.dense = torch.nn.Linear(64, 16)
    m = compress_model(Block(), PackRConfig(layer_scope="ffn", gradient_checkpointing=False))
    assert isinstance(m.intermediate.dense, PackRLinear) and isinstance(m.output.dense, PackRLinear)
    assert isinstance(m.attention.query, torch.nn.Linear)
    assert isinstance(m.attention.output.dense, torch.nn.Linear)  # attention output is not FFN
    m = compress_model(Block(), PackRConfig(layer_scope="attention", gradient_checkpointing=False))
    assert isinstance(m.attention.query, PackRLinear) and isinstance(m.intermediate.dense, torch.nn.Linear)
    m = compress_model(torch.nn.Sequential(torch.nn.Linear(8, 4)), PackRConfig(layer_scope="all", learnable_lut=False))
    assert isinstance(m[0], PackRLinear) and not m[0].lut.requires_grad


def test_api_surface_matches_reference():
    for name in ["PackRConfig", "PackRLinear", "PackRMatmulFunction", "packr_matmul", "compress_model", "SchemeType",
                 "FusedQuantizedAdam", "OffloadManager", "VelvetController", "PHRConfig", "PHRLinear",
                 "PHRMatmulFunction", "phr_matmul", "CV2LRTController"]:
        assert hasattr(packr, name), name
        assert name in packr.__all__, name
    assert packr.CV2LRTController is packr.VelvetController and packr.PHRLinear is PackRLinear
    with pytest.warns(RuntimeWarning):
        mgr = packr.OffloadManager(prefetch_depth=2)
    layer = PackRLinear(8, 4)
    mgr.register_wp("l0", layer.W_p)
    mgr.set_layer_sequence(["l0"])
    layer.attach_offload(mgr, "l0")
    mgr.prefetch_wp("l0"); mgr.ensure_wp("l0"); mgr.evict_wp("l0"); mgr.make_evict_cb("l0")()
    assert mgr.num_chunks == 0
    from packr_b200.cuda_adam import CUDA8BitAdam  # noqa: F401
    cfg = PackRConfig()
    assert (cfg.mode, cfg.layer_scope, cfg.block_size, cfg.optimizer_type) == ("packr", "ffn", 256, "triton8")


def test_compress_model_source_has_no_zstandard():
    import inspect
    from packr_b200.layer_patcher import compress_model as cm
    assert "zstandard" not in inspect.getsource(cm)


def test_gpu_ops_refuse_cpu_tensors():
    """No CPU fallback: the product path fails loudly on CPU tensors."""
    x = torch.randn(4, 64)
    W_p = torch.randint(0, 256, (64, 32), dtype=torch.uint8)
    W_f = torch.randn(64, 32, dtype=torch.bfloat16)
    lut = torch.randn(256)
    with pytest.raises(AssertionError):
        packr.packr_matmul(x, W_p, W_f, lut)
    layer = PackRLinear(64, 32)
    with pytest.raises(RuntimeError):
        layer(x)
    p = torch.nn.Parameter(torch.randn(10))
    p.grad = torch.randn(10)
    with pytest.raises(RuntimeError):
        packr.CUDA8BitAdam([p]).step()


def test_fused_quantized_adam_block_size():
    p = torch.nn.Parameter(torch.randn(10))
    with pytest.raises(ValueError):
        packr.FusedQuantizedAdam([p], block_size=128)
    packr.FusedQuantizedAdam([p], block_size=256, flat_buffer=True)
