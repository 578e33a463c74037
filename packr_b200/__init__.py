"""packr_b200 — PackR's training hot path on B200 (sm_100a).

Drop-in for the reference package's public surface on this path
(reference packr/__init__.py:13-45, packr/cuda_adam.py:142):

    import packr_b200 as packr
    from packr_b200 import compress_model, PackRConfig, PackRLinear
    from packr_b200.cuda_adam import CUDA8BitAdam

Every op runs hand-written sm_100a kernels from libpackr_b200.so through its
C ABI (include/packr_b200.h); there is no CPU fallback.
"""
from .cuda_adam import CUDA8BitAdam

__all__ = ["CUDA8BitAdam"]
