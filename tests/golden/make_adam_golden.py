"""Generates tests/golden/adam8_golden.npz by running the REFERENCE CUDA 8-bit
AdamW kernel (packr/cuda_adam_kernel.cu, compiled unmodified from the
reference tree into oracle/_ref/ref_adam8_cuda.so by oracle/build.py) on a
GPU, with the call sequence of reference packr/cuda_adam.py:160-192.

    python tests/golden/make_adam_golden.py [out.npz]      (needs a GPU)

Cases are small (ragged sizes, bf16 and fp32, with and without weight decay);
inputs come from packr_b200.synthetic seeds and are stored alongside the
reference's state after every step.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))
from packr_b200.synthetic import adam_grad, adam_params  # noqa: E402

CASES = {
    # name: (numel, dtype, lr, wd, grad std, steps)
    "bf16_ragged": (3 * 256 + 77, torch.bfloat16, 2e-5, 0.01, 1e-3, 6),
    "bf16_big_lr": (2048, torch.bfloat16, 1e-2, 0.0, 1e-1, 6),
    "f32_ragged": (5 * 256 + 3, torch.float32, 1e-3, 0.01, 1e-2, 6),
    "f32_tiny": (7, torch.float32, 2e-5, 0.0, 1e-3, 4),
}


def load_ref():
    so = REPO / "oracle" / "_ref" / "ref_adam8_cuda.so"
    spec = importlib.util.spec_from_file_location("ref_adam8_cuda", so)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def main() -> None:
    dst = Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).resolve().parent / "adam8_golden.npz"
    ref = load_ref()
    out = {}
    b1, b2, eps = 0.9, 0.999, 1e-8
    for name, (n, dt, lr, wd, gstd, steps) in CASES.items():
        p = adam_params(n, dtype=dt, seed=3, device="cuda")
        nb = (n + 255) // 256
        m = torch.zeros(n, dtype=torch.int8, device="cuda")
        v = torch.zeros(n, dtype=torch.int8, device="cuda")
        ms = torch.ones(nb, dtype=torch.float32, device="cuda")
        vs = torch.ones(nb, dtype=torch.float32, device="cuda")
        out[f"{name}/meta"] = np.array([n, int(dt == torch.bfloat16), steps], np.int64)
        out[f"{name}/hyper"] = np.array([lr, wd, gstd, b1, b2, eps], np.float64)
        out[f"{name}/p0"] = bits(p)
        for s in range(1, steps + 1):
            g = adam_grad(n, s, dtype=dt, device="cuda", std=gstd)
            out[f"{name}/g{s}"] = bits(g)
            bc1 = 1.0 - b1 ** s
            bc2 = 1.0 - b2 ** s
            ref.launch_adam_8bit(p, g, m, v, ms, vs, 1 if dt == torch.bfloat16 else 0, lr, b1, b2, eps, bc1, bc2, wd)
            torch.cuda.synchronize()
            for k, t in (("p", p), ("m", m), ("v", v), ("ms", ms), ("vs", vs)):
                out[f"{name}/{k}{s}"] = bits(t)
    dst.parent.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(dst, **out)
    print(dst, dst.stat().st_size)


if __name__ == "__main__":
    main()
