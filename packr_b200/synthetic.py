"""Seeded synthetic inputs for PackRLinear and the 8-bit AdamW step.

The workloads have no dataset: inputs are drawn from fixed seeds with the
shapes and value distributions of the benchmark configurations —
  x ~ N(0,1) (f32, or bf16 for the Llama-FFN shapes), W_p ~ U{0..255},
  lut = 256 sorted samples of N(0, 0.02*s), W_f = bf16(N(0, 0.002*s)),
  bias = bf16(N(0, 0.01)), upstream grad dY ~ N(0,1) (bf16-exact values when
  x is bf16), with s = sqrt(768/K) when scaled to fan-in;
  Adam: p = bf16(N(0, 0.02)), g = bf16(N(0, 1e-3)) freshly drawn per step.
Draw order from one torch.Generator: x, W_p, lut, W_f, bias, dY.
"""
from __future__ import annotations

import math

import torch


def linear_case(M: int, K: int, N: int, *, x_dtype=torch.float32, bias: bool = True, seed: int = 0,
                device="cpu", fanin_scaled: bool = False) -> dict:
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    s = math.sqrt(768.0 / K) if fanin_scaled else 1.0
    x = torch.randn(M, K, generator=g, device=dev).to(x_dtype)
    W_p = torch.randint(0, 256, (K, N), generator=g, device=dev, dtype=torch.uint8)
    lut = torch.sort(torch.randn(256, generator=g, device=dev) * (0.02 * s)).values.float()
    W_f = (torch.randn(K, N, generator=g, device=dev) * (0.002 * s)).to(torch.bfloat16)
    b = (torch.randn(N, generator=g, device=dev) * 0.01).to(torch.bfloat16) if bias else None
    dY = torch.randn(M, N, generator=g, device=dev)
    if x_dtype == torch.bfloat16:
        dY = dY.to(torch.bfloat16).float()
    return {"x": x, "W_p": W_p, "lut": lut, "W_f": W_f, "bias": b, "dY": dY}


def adam_params(n: int, *, dtype=torch.bfloat16, seed: int = 0, device="cpu") -> torch.Tensor:
    g = torch.Generator(device=torch.device(device)).manual_seed(seed)
    return (torch.randn(n, generator=g, device=device) * 0.02).to(dtype)


def adam_grad(n: int, step: int, *, dtype=torch.bfloat16, device="cpu", std: float = 1e-3) -> torch.Tensor:
    g = torch.Generator(device=torch.device(device)).manual_seed(1000 + step)
    return (torch.randn(n, generator=g, device=device) * std).to(dtype)
