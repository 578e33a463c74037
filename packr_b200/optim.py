"""FusedQuantizedAdam — the reference's Triton 8-bit AdamW class name
(reference packr/optim.py:80-389), served by the same sm_100a multi-tensor
kernel as CUDA8BitAdam.  Its Triton kernel and CPU step are not part of this
build; `block_size` must be 256 and `flat_buffer` is accepted (every group is
already one launch).  step() returns the closure's loss like the reference.
"""
from __future__ import annotations

import torch

from .cuda_adam import CUDA8BitAdam


class FusedQuantizedAdam(CUDA8BitAdam):
    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, block_size=256,
                 flat_buffer=False):
        if block_size != 256:
            raise ValueError("FusedQuantizedAdam: only block_size=256 is supported")
        super().__init__(params, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
        for g in self.param_groups:
            g.setdefault("block_size", block_size)
        self._flat_buffer = flat_buffer

    def enable_offload(self, manager):
        raise NotImplementedError("optimizer-state offload is not part of this build")

    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        super().step()
        return loss
