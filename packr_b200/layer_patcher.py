"""compress_model — replace nn.Linear layers by PackRLinear
(reference packr/layer_patcher.py:9-130, same name-based scope rules)."""
from __future__ import annotations

import warnings

import torch.nn as nn

from .config import PackRConfig
from .layer import PackRLinear


def compress_model(model: nn.Module, config: PackRConfig = None):
    """Replace nn.Linear layers of `model` with PackRLinear.  Returns the model."""
    if config is None:
        config = PackRConfig()
    if config.mode == "zpackr":
        raise NotImplementedError("mode='zpackr' is not available: its modules are absent from the reference tree")
    packr_layers = []
    for name, module in list(model.named_modules()):
        if not isinstance(module, nn.Linear):
            continue
        if not _matches_scope(name, config.layer_scope):
            continue
        packr = PackRLinear.from_linear(module)
        packr.lut.requires_grad_(config.learnable_lut)
        if name == "":  # the model itself is the Linear
            model = packr
        else:
            _replace_module(model, name, packr)
        packr_layers.append((name, packr))
    if config.gradient_checkpointing:
        _enable_gradient_checkpointing(model)
    if config.offload and packr_layers:
        warnings.warn("PackRConfig.offload is ignored: this build keeps W_p and the optimizer state in HBM",
                      stacklevel=2)
    return model


def _replace_module(model, name, new_module):
    parent = model
    parts = name.split(".")
    for part in parts[:-1]:
        parent = getattr(parent, part)
    setattr(parent, parts[-1], new_module)


def _matches_scope(name: str, scope: str) -> bool:
    if scope == "all":
        return True
    if scope == "ffn":
        return _is_ffn(name)
    if scope == "attention":
        return _is_attention(name) and not _is_ffn(name)
    return False


def _is_ffn(name: str) -> bool:
    ffn_intermediate = ["intermediate", "fc1", "mlp.up", "ffn.up", "dense_h_to_4h"]
    ffn_output = ["output.dense", "fc2", "mlp.down", "ffn.down", "dense_4h_to_h"]
    n = name.lower()
    if any(m in n for m in ffn_intermediate):
        return True
    if any(m in n for m in ffn_output) and "attention" not in n:
        return True
    return False


def _is_attention(name: str) -> bool:
    attn = ["query", "key", "value", "q_proj", "k_proj", "v_proj", "o_proj", "out_proj"]
    n = name.lower()
    return any(m in n for m in attn)


def _enable_gradient_checkpointing(model: nn.Module):
    try:
        model.gradient_checkpointing_enable()
    except AttributeError:
        pass
