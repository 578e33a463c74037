"""Model-level workloads of the hot path (synthetic data, random init): the
BERT-base fine-tune step with compressed FFN layers and the Llama-3-8B-shaped
decoder with every Linear compressed.  Used by bench.py and the GPU tests;
the model code itself is transformers' (BertForSequenceClassification,
LlamaForCausalLM), only its Linear layers are replaced.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .config import PackRConfig
from .layer import PackRLinear
from .layer_patcher import compress_model

BERT_BASE = dict(vocab_size=30522, hidden_size=768, num_hidden_layers=12, num_attention_heads=12,
                 intermediate_size=3072)
LLAMA3_8B = dict(vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                 num_attention_heads=32, num_key_value_heads=8)


def bert_classifier(device, layers: int = 12, seed: int = 0, **overrides):
    """BertForSequenceClassification (2 labels, fp32) with its FFN Linear
    layers compressed by compress_model(layer_scope="ffn") (from_linear)."""
    from transformers import BertConfig, BertForSequenceClassification
    torch.manual_seed(seed)
    cfg = BertConfig(**{**BERT_BASE, "num_hidden_layers": layers, **overrides}, num_labels=2)
    model = BertForSequenceClassification(cfg).to(device)
    compress_model(model, PackRConfig(layer_scope="ffn"))
    return model


def bert_batch(device, batch: int = 32, seq: int = 128, vocab: int = 30522, seed: int = 0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    ids = torch.randint(0, vocab, (batch, seq), generator=g).to(device)
    labels = torch.randint(0, 2, (batch,), generator=g).to(device)
    return ids, labels


class _Cast(nn.Module):
    """PackRLinear whose f32 output (the reference's dtype) is cast to the
    activation dtype of a bf16 model."""

    def __init__(self, inner: PackRLinear, dtype: torch.dtype):
        super().__init__()
        self.inner = inner
        self.dtype = dtype

    def forward(self, x):
        return self.inner(x).to(self.dtype)


def llama_decoder(device, layers: int = 32, seed: int = 0, dtype=torch.bfloat16, **overrides):
    """LlamaForCausalLM (Llama-3-8B shapes by default) in bf16 with every
    Linear, lm_head included, replaced by a synthetic-init PackRLinear (W_p
    uniform, sorted N(0, 0.02 sqrt(768/K)) lut, N(0, 0.002 sqrt(768/K)) W_f)
    whose output is cast back to bf16."""
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(seed)
    cfg = LlamaConfig(**{**LLAMA3_8B, "num_hidden_layers": layers, **overrides})
    cfg.max_position_embeddings = 4096
    prev = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        with torch.device(device):
            model = LlamaForCausalLM(cfg)  # its bf16 Linear weights are freed below
    finally:
        torch.set_default_dtype(prev)
    names = [n for n, m in model.named_modules() if isinstance(m, nn.Linear)]
    for i, name in enumerate(names):
        lin = model.get_submodule(name)
        pk = PackRLinear.synthetic(lin.in_features, lin.out_features, bias=lin.bias is not None, device=device,
                                   seed=seed * 100003 + i,
                                   lut_std=0.02 * (768 / lin.in_features) ** 0.5,
                                   wf_std=0.002 * (768 / lin.in_features) ** 0.5)
        parent, _, leaf = name.rpartition(".")
        setattr(model.get_submodule(parent) if parent else model, leaf, _Cast(pk, dtype))
        del lin
    if device != "cpu":
        torch.cuda.empty_cache()
    return model


def llama_batch(device, seq: int = 2048, batch: int = 1, vocab: int = 128256, seed: int = 0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    ids = torch.randint(0, vocab, (batch, seq), generator=g).to(device)
    return ids
