"""Autograd for the PackR linear map on B200.

PackRLinearFunction: out = x @ (W_f + lut[W_p]) + bias, with the bias fused
into the forward GEMM's epilogue and its gradient produced by the backward
launch sequence.  Backward semantics follow reference packr/autograd.py:56-88:
  grad_x    = bf16(bf16(dY) @ W_bf16^T), returned in x's dtype
  grad_W_f  = bf16(x^T @ dY)                  (fp32 accumulate)
  grad_lut  = scatter_add(x^T @ dY by W_p) / (bincount(W_p) + 1e-8)
  grad_bias = bf16(dY.sum(0))                 (autograd of layer.py:97)
W_p is frozen and gets no gradient.

PackRMatmulFunction keeps the reference's signature
(x, W_p, W_f, lut, evict_cb=None, layer_name=None, offload_mgr=None) and
bias-free output (reference autograd.py:17-53).  Host offload is not part of
this build (W_p stays in HBM), so layer_name / offload_mgr are accepted and
ignored; evict_cb still fires at the end of backward.
"""
from __future__ import annotations

import os

import torch

from . import kernel as _k

# Off by default: between forward and backward a layer holds only its packed
# weights (3 bytes per weight), as PackR promises.  PACKR_KEEP_DECODED_W=1
# trades 2 more bytes per weight, held from forward to backward on the
# many-row route, for the second decode of W in the backward.
KEEP_DECODED_W = os.environ.get("PACKR_KEEP_DECODED_W", "0") == "1"


def grad_sink(param: torch.Tensor) -> torch.Tensor | None:
    """A fresh view of the gradient buffer an optimizer registered for
    `param` (param._packr_grad_sink = (flat_buffer, element_offset)), or None.
    Only offered while param.grad is None: the backward then writes the
    gradient straight into the buffer and autograd adopts the view as
    param.grad without a copy; with a gradient already present, autograd
    accumulates into it as usual."""
    if param is None or param.grad is not None:
        return None
    spec = getattr(param, "_packr_grad_sink", None)
    if spec is None:
        return None
    buf, off = spec
    n = param.numel()
    if buf.dtype != param.dtype or buf.device != param.device or off + n > buf.numel():
        return None
    return buf[off:off + n].view(param.shape)


def _forward_keep_w(ctx, x, W_p, W_f, lut, bias):
    """The forward; on the route where it decodes all of W first (many rows)
    and dX will be needed, the decoded W is kept on ctx for the backward's
    dX GEMM (2 bytes per weight held until the backward), so W is decoded
    once per step instead of twice."""
    ctx.wd = None
    x2 = x.reshape(-1, x.shape[-1]) if x.dim() != 2 else x
    M, K = x2.shape
    N = W_p.shape[1]
    if KEEP_DECODED_W and ctx.needs_input_grad[0] and _k.predecode_route(M, K, N, W_p, W_f):
        ctx.wd = _k.predecode_bf16(W_p, W_f, lut)
        return _k.forward_decoded(x, ctx.wd, bias)
    return _k.forward(x, W_p, W_f, lut, bias)


class PackRLinearFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, W_p, W_f, lut, bias=None, counts=None, evict_cb=None):
        if not x.is_cuda:
            raise RuntimeError("PackRLinear runs on CUDA tensors only (no CPU path in the B200 build)")
        ctx.save_for_backward(x, W_p, W_f, lut, counts)
        ctx.has_bias = bias is not None
        ctx.evict_cb = evict_cb
        ctx.wf_param = W_f
        return _forward_keep_w(ctx, x, W_p, W_f, lut, bias)

    @staticmethod
    def backward(ctx, grad_out):
        x, W_p, W_f, lut, counts = ctx.saved_tensors
        nx, _, nwf, nlut, nb = ctx.needs_input_grad[:5]
        dX, dW, dlut, dbias = _k.backward(grad_out, x, W_p, W_f, lut, counts, need_dx=nx, need_dw=nwf,
                                          need_dlut=nlut, need_dbias=ctx.has_bias and nb,
                                          dW_out=grad_sink(ctx.wf_param) if nwf else None,
                                          Wd=ctx.wd if nx else None)
        ctx.wd = None
        if ctx.evict_cb is not None:
            ctx.evict_cb()
        if dX is not None and dX.dtype != x.dtype:
            dX = dX.to(x.dtype)
        return dX, None, dW, dlut, dbias, None, None


class PackRMatmulFunction(torch.autograd.Function):
    """Custom autograd for out = x @ (W_f + lut[W_p]) (bias handled outside),
    reference packr/autograd.py:17-88."""

    @staticmethod
    def forward(ctx, x, W_p, W_f, lut, evict_cb=None, layer_name=None, offload_mgr=None):
        ctx.save_for_backward(x, W_p, W_f, lut)
        ctx._evict_cb = evict_cb
        ctx.wf_param = W_f
        return _k.packr_matmul(x, W_p, W_f, lut)

    @staticmethod
    def backward(ctx, grad_out):
        x, W_p, W_f, lut = ctx.saved_tensors
        nx, _, nwf, nlut = ctx.needs_input_grad[:4]
        dX, dW, dlut, _ = _k.backward(grad_out, x, W_p, W_f, lut, None, need_dx=nx, need_dw=nwf, need_dlut=nlut,
                                      need_dbias=False, dW_out=grad_sink(ctx.wf_param) if nwf else None)
        if ctx._evict_cb is not None:
            ctx._evict_cb()
        if dX is not None and dX.dtype != x.dtype:
            dX = dX.to(x.dtype)
        return dX, None, dW, dlut, None, None, None


# Legacy alias (reference packr/__init__.py:32)
PHRMatmulFunction = PackRMatmulFunction
