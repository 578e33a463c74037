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

        The compression always runs in the library's kernels (exact order
        statistics for the quantile, one encode pass; no size limit), on the
        weight's own GPU or, for a weight held in host memory, on the current
        CUDA device, after which the new layer's tensors are moved back to
        the weight's device, as the reference leaves them there.  f32, bf16
        and f16 weights give the reference's results bit for bit (W * scale
        rounded to the weight's type with the multiplier torch uses on the
        weight's device); a weight of another dtype (f64) is compressed from
        its values rounded to f32."""
        if not isinstance(module, nn.Linear):
            raise TypeError(f"Expected nn.Linear, got {type(module)}")
        w = module.weight.detach()
        home = w.device
        if not w.is_cuda:
            if not torch.cuda.is_available():
                raise RuntimeError("PackRLinear.from_linear compresses on a CUDA device; none is available "
                                   "(the B200 build has no CPU path)")
            w = w.to(torch.device("cuda", torch.cuda.current_device()))
        if w.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            w = w.float()
        m = cls._from_linear_cuda(w, module.bias, home)
        return m if home.type == "cuda" else m.to(home)

    @classmethod
    def _from_linear_cuda(cls, w: torch.Tensor, bias: torch.Tensor | None, home: torch.device):
        from . import kernel
        device = w.device
        out_f, in_f = w.shape
        # the scalar arithmetic on the weight's own device, as the reference;
        # |f16| values are exact in f32, which the order statistics read
        q99 = kernel.quantile_abs(w if w.dtype != torch.float16 else w.float(), 0.99, home) + 1e-6
        scale = 1.6 / q99
        # W_orig * scale for a 16-bit weight: the multiplier as torch applies
        # it on the weight's own device, where the reference computes it
        half = w.dtype in (torch.bfloat16, torch.float16)
        target_scale = kernel.half_product_multiplier(scale, w.dtype, home) if half else scale
        W_p, W_f, lut = kernel.from_linear_encode(w, _build_codebook().to(device), scale, target_scale)
        m = cls.__new__(cls)
        nn.Module.__init__(m)
        m.in_features, m.out_features = in_f, out_f
        m.W_p = nn.Parameter(W_p, requires_grad=False)
        m.W_f = nn.Parameter(W_f)
        m.lut = nn.Parameter(lut)
        m.bias_f = (nn.Parameter(bias.detach().to(device=device, dtype=torch.bfloat16).clone())
                    if bias is not None else None)
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
