"""PackRLinear — packed-residual linear layer on B200.

Drop-in for reference packr/layer.py:41-159: same constructor, parameters
  W_p    uint8 [in, out]  frozen byte indices (requires_grad=False)
  W_f    bf16  [in, out]  trainable residual
  lut    f32   [256]      trainable lookup table
  bias_f bf16  [out]      optional
and `from_linear`.  forward() flattens 3-D input as the reference does
(layer.py:79-81, 99-100); the bias add of layer.py:96-97 is fused into the
GEMM epilogue, and the lut bin counts used by the lut gradient are cached per
layer (W_p is frozen) instead of recounted every backward.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .autograd import PackRLinearFunction
from . import kernel as _k


def _build_codebook() -> torch.Tensor:
    """256-entry codebook (reference layer.py:24-38): byte i encodes gain
    nibble g = i & 15 -> (g - 7.5)/7.5 and scale nibble s = i >> 4 -> (s+1)/10;
    codebook[i] = gain * scale."""
    i = torch.arange(256, dtype=torch.float64)
    g = torch.remainder(i, 16)
    s = torch.floor(i / 16)
    return (((g - 7.5) / 7.5) * ((s + 1.0) / 10.0)).to(torch.float32)


def _quantile_abs(w: torch.Tensor, q: float) -> torch.Tensor:
    """torch.quantile(|w|, q) (linear interpolation), also for tensors above
    torch.quantile's 2^24-element limit (exact order statistics by kthvalue)."""
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


class PackRLinear(nn.Module):
    """PackR linear layer with learnable LUT: out = x @ (W_f + lut[W_p]) + bias."""

    def __init__(self, in_features, out_features, bias=True):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.W_p = nn.Parameter(torch.randint(0, 256, (in_features, out_features), dtype=torch.uint8),
                                requires_grad=False)
        self.W_f = nn.Parameter(torch.randn(in_features, out_features, dtype=torch.bfloat16) * 0.02)
        self.lut = nn.Parameter(torch.zeros(256, dtype=torch.float32))
        self.bias_f = nn.Parameter(torch.zeros(out_features, dtype=torch.bfloat16)) if bias else None
        self._counts = None
        self._counts_key = None
        self._offload_mgr = None
        self._layer_name = None

    def attach_offload(self, manager, layer_name):
        """Kept for API compatibility (reference layer.py:68-76).  This build
        keeps W_p resident in HBM; the manager is recorded but not used."""
        self._offload_mgr = manager
        self._layer_name = layer_name

    def lut_counts(self) -> torch.Tensor:
        """bincount(W_p, 256) as int32, cached until W_p changes."""
        w = self.W_p
        key = (w.data_ptr(), w._version, w.device)
        if self._counts is None or self._counts_key != key:
            self._counts = _k.bincount256(w.detach())
            self._counts_key = key
        return self._counts

    def forward(self, x):
        if not (x.is_cuda and self.W_p.is_cuda):
            raise RuntimeError("PackRLinear runs on CUDA tensors only (no CPU path in the B200 build)")
        orig_shape = x.shape
        if x.dim() == 3:
            x = x.reshape(-1, x.shape[-1])
        counts = self.lut_counts() if self.lut.requires_grad else None
        out = PackRLinearFunction.apply(x, self.W_p, self.W_f, self.lut, self.bias_f, counts)
        if len(orig_shape) == 3:
            out = out.reshape(orig_shape[0], orig_shape[1], -1)
        return out

    def extra_repr(self):
        return f"in_features={self.in_features}, out_features={self.out_features}, bias={self.bias_f is not None}"

    @classmethod
    def from_linear(cls, module: nn.Linear):
        """Convert an nn.Linear (reference layer.py:106-159): scale |W| so its
        99th percentile maps to 1.6, take the nearest codebook entry per weight
        (lowest index on ties), lut = codebook / scale, W_f = W - lut[W_p].

        A CUDA f32/bf16 weight is compressed by the library's kernels (exact
        order statistics for the quantile, one encode pass; no size limit);
        other weights by the same torch operations as the reference."""
        if not isinstance(module, nn.Linear):
            raise TypeError(f"Expected nn.Linear, got {type(module)}")
        if module.weight.is_cuda and module.weight.dtype in (torch.float32, torch.bfloat16):
            return cls._from_linear_cuda(module)
        return cls._from_linear_torch(module)

    @classmethod
    def _from_linear_torch(cls, module: nn.Linear):
        """The reference's torch operation sequence (any device)."""
        packr = cls(module.in_features, module.out_features, bias=module.bias is not None)
        device = module.weight.device
        codebook = _build_codebook().to(device)
        W_orig = module.weight.detach().t()
        q99 = _quantile_abs(W_orig, 0.99) + 1e-6
        scale = 1.6 / q99
        W_target = torch.clamp(W_orig * scale, -1.6, 1.6)
        in_f, out_f = W_orig.shape
        best = torch.empty(in_f, out_f, dtype=torch.uint8, device=device)
        cb = codebook.view(1, 1, 256)
        # chunk rows so the [rows, out, 256] distance temporary stays ~256 MB
        chunk = max(1, min(256, (1 << 26) // max(out_f * 256, 1)))
        for s in range(0, in_f, chunk):
            e = min(s + chunk, in_f)
            diff = torch.abs(W_target[s:e].unsqueeze(-1) - cb)
            best[s:e] = torch.argmin(diff, dim=-1).to(torch.uint8)
        dequant_lut = codebook / scale
        quantized = dequant_lut[best.long()]
        packr.W_p.data = best.contiguous()
        packr.lut.data = dequant_lut.contiguous().to(device=device, dtype=torch.float32)
        packr.W_f.data = (W_orig - quantized).contiguous().to(device=device, dtype=torch.bfloat16)
        if module.bias is not None:
            packr.bias_f.data = module.bias.detach().to(device=device, dtype=torch.bfloat16)
        return packr

    @classmethod
    def _from_linear_cuda(cls, module: nn.Linear):
        from . import kernel
        w = module.weight.detach()
        device = w.device
        in_f, out_f = module.in_features, module.out_features
        q99 = kernel.quantile_abs(w, 0.99) + 1e-6
        scale = 1.6 / q99
        # W_orig * scale for a bf16 weight: the multiplier as torch applies it
        target_scale = kernel.bf16_product_multiplier(scale) if w.dtype == torch.bfloat16 else scale
        W_p, W_f, lut = kernel.from_linear_encode(w, _build_codebook().to(device), scale, target_scale)
        m = cls.__new__(cls)
        nn.Module.__init__(m)
        m.in_features, m.out_features = in_f, out_f
        m.W_p = nn.Parameter(W_p, requires_grad=False)
        m.W_f = nn.Parameter(W_f)
        m.lut = nn.Parameter(lut)
        m.bias_f = (nn.Parameter(module.bias.detach().to(device=device, dtype=torch.bfloat16).clone())
                    if module.bias is not None else None)
        m._counts = None
        m._counts_key = None
        m._offload_mgr = None
        m._layer_name = None
        return m

    @classmethod
    def synthetic(cls, in_features, out_features, bias=True, *, device="cuda", seed=0, lut_std=0.02,
                  wf_std=0.002, dtype_bias=torch.bfloat16):
        """A PackRLinear with seeded synthetic parameters (uniform W_p,
        sorted N(0, lut_std) lut, N(0, wf_std) W_f), built directly on
        `device` — the initialisation of the large benchmark models, which
        skip the nearest-codebook search of from_linear."""
        g = torch.Generator(device=device).manual_seed(seed)
        m = cls.__new__(cls)
        nn.Module.__init__(m)
        m.in_features, m.out_features = in_features, out_features
        m.W_p = nn.Parameter(torch.randint(0, 256, (in_features, out_features), generator=g, device=device,
                                           dtype=torch.uint8), requires_grad=False)
        m.lut = nn.Parameter(torch.sort(torch.randn(256, generator=g, device=device) * lut_std).values)
        m.W_f = nn.Parameter((torch.randn(in_features, out_features, generator=g, device=device) * wf_std)
                             .to(torch.bfloat16))
        m.bias_f = nn.Parameter(torch.zeros(out_features, device=device, dtype=dtype_bias)) if bias else None
        m._counts = None
        m._counts_key = None
        m._offload_mgr = None
        m._layer_name = None
        return m


# Legacy alias
PHRLinear = PackRLinear
