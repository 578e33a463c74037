"""Configuration for PackR memory-efficient training (reference packr/config.py:11-45).

Same fields and defaults.  In this build `offload` and mode "zpackr" are not
available (host offload is unnecessary at B200 memory sizes and the zpackr
modules are not part of the reference tree); `compress_model` reports them.
`use_8bit_optimizer` / `optimizer_type` are advisory, as in the reference:
the caller constructs the optimizer.
"""
from dataclasses import dataclass
from typing import Literal

SchemeType = Literal["phr"]
ModeType = Literal["packr", "zpackr"]


@dataclass
class PackRConfig:
    mode: ModeType = "packr"
    scheme: SchemeType = "phr"
    learnable_lut: bool = True
    layer_scope: Literal["ffn", "attention", "all"] = "ffn"
    gradient_checkpointing: bool = True
    use_8bit_optimizer: bool = True
    offload: bool = False
    block_size: int = 256
    bf16: bool = False
    hash_interval: int = 1
    optimizer_type: Literal["triton8", "cuda8", "adamw"] = "triton8"
    gradient_mix: float = 0.5
    grad_ema_beta: float = 0.9967


# Legacy alias
PHRConfig = PackRConfig
