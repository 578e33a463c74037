"""CUDA8BitAdam — 8-bit AdamW with per-block int8 moments on sm_100a.

Drop-in for reference packr/cuda_adam.py:142-194: same constructor, same
`step(closure=None)`, same lazily created per-parameter state
  state[p]["m"], ["v"]              int8  [numel]
  state[p]["m_scale"], ["v_scale"]  f32   [ceil(numel/256)]  (init ones)
(reference packr/cuda_adam.py:132-139), which VelvetController reads.
Instead of one kernel launch per parameter, each parameter group is updated
by one packr_adam8_multi call (libpackr_b200.so), which walks every tensor of
the group with 128-bit vector accesses.

Additions over the reference: `_step_count` is saved in state_dict() (the
reference keeps it only as an attribute, so bias correction restarted on
resume), load_state_dict() keeps the int8 codes and f32 scales of bf16
parameters in their dtypes (torch's loader casts them to bf16), and step()
raises if a parameter is not on a CUDA device.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

BLOCK_SIZE = 256


def _init_state(state, p):
    """Initialise int8 m/v + per-block float32 scales for one param
    (reference packr/cuda_adam.py:132-139)."""
    n = p.numel()
    nb = (n + BLOCK_SIZE - 1) // BLOCK_SIZE
    state["m"] = torch.zeros(n, dtype=torch.int8, device=p.device)
    state["v"] = torch.zeros(n, dtype=torch.int8, device=p.device)
    state["m_scale"] = torch.ones(nb, dtype=torch.float32, device=p.device)
    state["v_scale"] = torch.ones(nb, dtype=torch.float32, device=p.device)


def selfcheck_rounding(device="cuda") -> list[int]:
    """Mismatch counts of the kernel's short correctly rounded sequences
    against CUDA's IEEE operations on `device` (packr_selfcheck_rounding):
    [reciprocals, square roots, quotients, whole updates]; all 0 when the
    device computes them exactly."""
    lib = _lib.load()
    dev = torch.device(device)
    out = torch.empty(4, dtype=torch.int64, device=dev)
    with torch.cuda.device(dev):
        code = lib.packr_selfcheck_rounding(ctypes.c_void_p(out.data_ptr()),
                                            ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    _lib.check("packr_selfcheck_rounding", code)
    return [int(v) for v in out.cpu().tolist()]


def _adam_tensors(entries):
    """ctypes packr_adam_tensor array of `entries` and their device."""
    arr = (_lib.AdamTensor * len(entries))()
    dev = None
    for i, (p, g, m, v, ms, vs) in enumerate(entries):
        if not p.is_cuda:
            raise RuntimeError("CUDA8BitAdam: parameters must be CUDA tensors (no CPU path)")
        if dev is None:
            dev = p.device
        elif p.device != dev:
            raise RuntimeError("adam8_launch: all tensors of one launch must be on one device")
        if g.dtype != p.dtype or p.dtype not in (torch.bfloat16, torch.float32):
            raise TypeError(f"CUDA8BitAdam: unsupported dtype {p.dtype}/{g.dtype}")
        for t in (p, g, m, v, ms, vs):
            if not t.is_contiguous():
                raise ValueError("adam8_launch: tensors must be contiguous")
        e = arr[i]
        e.p, e.g, e.m, e.v = p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr()
        e.m_scale, e.v_scale = ms.data_ptr(), vs.data_ptr()
        e.numel = p.numel()
        e.dtype = _lib.PACKR_DTYPE_BF16 if p.dtype == torch.bfloat16 else _lib.PACKR_DTYPE_F32
        e.reserved = 0
    return arr, dev


def adam8_launch(entries, lr, b1, b2, eps, bc1, bc2, wd, stream=None) -> None:
    """Runs packr_adam8_multi over `entries` = [(p, g, m, v, ms, vs), ...] of
    CUDA tensors on one device.  p/g are bf16 or f32 (same dtype), contiguous."""
    if not entries:
        return
    lib = _lib.load()
    arr, dev = _adam_tensors(entries)
    with torch.cuda.device(dev):
        s = stream if stream is not None else torch.cuda.current_stream(dev)
        code = lib.packr_adam8_multi(arr, len(entries), lr, b1, b2, eps, bc1, bc2, wd,
                                     ctypes.c_void_p(s.cuda_stream))
    _lib.check("packr_adam8_multi", code)


def adam8_launch_push(entries, peer_ptrs, lr, b1, b2, eps, bc1, bc2, wd, stream=None) -> None:
    """adam8_launch that also stores entry i's updated values at each device
    address in peer_ptrs[i] (the same tensor in other GPUs' memory, mapped
    with packr_ipc_open; every entry has the same number of peers, at most 7)
    through packr_adam8_multi_push."""
    if not entries:
        return
    n_peers = len(peer_ptrs[0]) if peer_ptrs else 0
    if len(peer_ptrs) != len(entries) or any(len(q) != n_peers for q in peer_ptrs):
        raise ValueError("adam8_launch_push: one list of peer addresses per entry, all of one length")
    lib = _lib.load()
    arr, dev = _adam_tensors(entries)
    flat = (ctypes.c_void_p * max(len(entries) * n_peers, 1))(*[a for q in peer_ptrs for a in q])
    with torch.cuda.device(dev):
        s = stream if stream is not None else torch.cuda.current_stream(dev)
        code = lib.packr_adam8_multi_push(arr, len(entries), flat, n_peers, lr, b1, b2, eps, bc1, bc2, wd,
                                          ctypes.c_void_p(s.cuda_stream))
    _lib.check("packr_adam8_multi_push", code)


class CUDA8BitAdam(torch.optim.Optimizer):
    """8-bit AdamW with per-block int8 quantization (block 256).

    Args:
        params:       iterable of parameters (bf16 or fp32, CUDA)
        lr:           learning rate
        betas:        (beta1, beta2)
        eps:          epsilon
        weight_decay: AdamW-style weight decay
    """

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0):
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
        super().__init__(params, defaults)
        self._step_count = 0

    @torch.no_grad()
    def step(self, closure=None):
        if closure is not None:
            with torch.enable_grad():
                closure()
        self._step_count += 1
        step = self._step_count
        for group in self.param_groups:
            lr = group["lr"]
            b1, b2 = group["betas"]
            eps = group["eps"]
            wd = group["weight_decay"]
            bc1 = 1.0 - b1 ** step
            bc2 = 1.0 - b2 ** step
            by_dev = {}
            for p in group["params"]:
                if p.grad is None:
                    continue
                if p.grad.is_sparse:
                    raise RuntimeError("CUDA8BitAdam does not support sparse gradients")
                state = self.state[p]
                if "m" not in state:
                    _init_state(state, p)
                g = p.grad if p.grad.is_contiguous() else p.grad.contiguous()
                if g.dtype != p.dtype:
                    g = g.to(p.dtype)
                if not p.is_contiguous():
                    raise ValueError("CUDA8BitAdam: parameters must be contiguous")
                by_dev.setdefault(p.device, []).append(
                    (p, g, state["m"], state["v"], state["m_scale"], state["v_scale"]))
            for entries in by_dev.values():
                adam8_launch(entries, lr, b1, b2, eps, bc1, bc2, wd)
        return None

    def state_dict(self):
        sd = super().state_dict()
        sd["packr_step_count"] = self._step_count
        return sd

    def load_state_dict(self, state_dict):
        """torch's Optimizer.load_state_dict casts every state tensor of a
        floating-point parameter to the parameter's dtype, which would turn
        the int8 codes and the f32 block scales of a bf16 parameter into
        bf16; the 8-bit state is put back with its own dtypes."""
        state_dict = dict(state_dict)
        self._step_count = int(state_dict.pop("packr_step_count", self._step_count))
        super().load_state_dict(state_dict)
        saved = [i for g in state_dict["param_groups"] for i in g["params"]]
        params = [p for g in self.param_groups for p in g["params"]]
        for idx, p in zip(saved, params):
            st = state_dict["state"].get(idx)
            if not st:
                continue
            for k in ("m", "v", "m_scale", "v_scale"):
                if k in st:
                    self.state[p][k] = st[k].detach().to(device=p.device).clone()
