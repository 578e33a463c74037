"""Torch restatement of the reference PackRLinear forward + backward and of
its from_linear conversion — TEST / BASELINE INFRASTRUCTURE ONLY (tests/ and
__graft_entry__.smoke() use it as the checker, bench.py's CPU legs time it).

Line for line the reference's CPU-capable arithmetic:
  forward   packr/kernel.py:127-139  decoded = fp16(lut[W_p]); w_full = W_f + decoded
                                     (fp32 by promotion); out = x.float() @ w_full
  backward  packr/autograd.py:65-83  Wb = W_f + bf16(lut[W_p]); dX = (bf16(dY) @ Wb.T).float();
                                     dW = x.T.float() @ dY.float(); grad_W_f = bf16(dW);
                                     counts = bincount(W_p); dlut = scatter_add(dW)/(counts+1e-8)
  from_linear packr/layer.py:117-157 quantile, nearest codebook entry, residual
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


# --------------------------------------------------------------------------
# from_linear (packr/layer.py:24-38 codebook, 106-159 conversion)
# --------------------------------------------------------------------------


def codebook() -> torch.Tensor:
    """The 256-entry codebook of packr/layer.py:24-38: byte i holds gain
    nibble g = i & 15 -> (g - 7.5) / 7.5 and scale nibble s = i >> 4 ->
    (s + 1) / 10; entry i = gain * scale (computed in f64, stored f32)."""
    i = torch.arange(256, dtype=torch.float64)
    g = torch.remainder(i, 16)
    s = torch.floor(i / 16)
    return (((g - 7.5) / 7.5) * ((s + 1.0) / 10.0)).to(torch.float32)


def quantile_abs(w: torch.Tensor, q: float) -> torch.Tensor:
    """torch.quantile(|w|.float(), q) as packr/layer.py:128 computes it; for
    tensors above torch.quantile's 2^24-element limit (where the reference
    raises) the same linear interpolation between the two exact order
    statistics, found by kthvalue."""
    a = w.abs().float().reshape(-1)
    n = a.numel()
    if n <= (1 << 24):
        return torch.quantile(a, q)
    pos = torch.tensor(q, dtype=torch.float32) * (n - 1)
    lo = int(torch.floor(pos).item())
    hi = min(lo + 1, n - 1)
    v_lo = torch.kthvalue(a, lo + 1).values
    v_hi = torch.kthvalue(a, hi + 1).values if hi != lo else v_lo
    return torch.lerp(v_lo, v_hi, (pos - lo).to(a.device))


def from_linear(weight: torch.Tensor, bias: torch.Tensor | None = None) -> dict:
    """The reference's nn.Linear -> PackRLinear conversion (packr/layer.py:
    117-157), op for op on the weight's own device: q99 = quantile(|W|) +
    1e-6, scale = 1.6 / q99, target = clamp(W * scale, +-1.6), W_p = argmin
    over the codebook of |target - codebook| (torch.argmin: lowest index on
    ties; rows chunked so the distance temporary stays ~256 MB), lut =
    codebook / scale, W_f = bf16(W - lut[W_p]), bias_f = bf16(bias).
    `weight` is nn.Linear's [out, in]; returns W_p u8 / W_f bf16 [in, out],
    lut f32 [256] and bias_f (or None)."""
    device = weight.device
    cb = codebook().to(device)
    W_orig = weight.detach().t()
    q99 = quantile_abs(W_orig, 0.99) + 1e-6
    scale = 1.6 / q99
    W_target = torch.clamp(W_orig * scale, -1.6, 1.6)
    in_f, out_f = W_orig.shape
    best = torch.empty(in_f, out_f, dtype=torch.uint8, device=device)
    cb3 = cb.view(1, 1, 256)
    chunk = max(1, min(256, (1 << 26) // max(out_f * 256, 1)))
    for s in range(0, in_f, chunk):
        e = min(s + chunk, in_f)
        best[s:e] = torch.argmin(torch.abs(W_target[s:e].unsqueeze(-1) - cb3), dim=-1).to(torch.uint8)
    lut = cb / scale
    quantized = lut[best.long()]
    return {"W_p": best.contiguous(), "lut": lut.contiguous().to(torch.float32),
            "W_f": (W_orig - quantized).contiguous().to(torch.bfloat16),
            "bias_f": None if bias is None else bias.detach().to(torch.bfloat16)}
