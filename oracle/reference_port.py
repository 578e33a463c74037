"""Torch-CPU restatement of the reference PackRLinear forward + backward —
TEST / BASELINE INFRASTRUCTURE ONLY (bench.py's CPU legs time it).

Line for line the reference's CPU-capable arithmetic:
  forward   packr/kernel.py:127-139  decoded = fp16(lut[W_p]); w_full = W_f + decoded
                                     (fp32 by promotion); out = x.float() @ w_full
  backward  packr/autograd.py:65-83  Wb = W_f + bf16(lut[W_p]); dX = (bf16(dY) @ Wb.T).float();
                                     dW = x.T.float() @ dY.float(); grad_W_f = bf16(dW);
                                     counts = bincount(W_p); dlut = scatter_add(dW)/(counts+1e-8)
using torch's CPU kernels with all host threads, as the reference does when
run on a CPU (its own decode fallback is _kernel_loader._fallback_decode).
"""
from __future__ import annotations

import torch


def forward(x, W_p, W_f, lut):
    decoded = lut[W_p.long()].to(torch.float16)
    w_full = W_f + decoded
    return x.float() @ w_full if x.dtype != w_full.dtype else x @ w_full


def backward(grad_out, x, W_p, W_f, lut):
    w_full_bf16 = W_f + lut[W_p.long()].to(torch.bfloat16)
    grad_x = (grad_out.to(torch.bfloat16) @ w_full_bf16.T).float()
    dW_full = x.T.float() @ grad_out.float()
    grad_w_f = dW_full.to(W_f.dtype)
    flat = W_p.flatten().long()
    counts = torch.bincount(flat, minlength=256).float()
    grad_lut = torch.zeros(256, dtype=torch.float32)
    grad_lut.scatter_add_(0, flat, dW_full.flatten())
    grad_lut /= counts + 1e-8
    return grad_x.to(x.dtype), grad_w_f, grad_lut
