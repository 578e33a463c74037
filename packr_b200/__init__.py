"""packr_b200 — PackR's training hot path on B200 (sm_100a).

Drop-in for the reference package's public surface on this path
(reference packr/__init__.py:13-45, packr/cuda_adam.py:142):

    import packr_b200 as packr
    from packr_b200 import compress_model, PackRConfig, PackRLinear, VelvetController
    from packr_b200.cuda_adam import CUDA8BitAdam

Every op runs hand-written sm_100a kernels from libpackr_b200.so through its
C ABI (include/packr_b200.h); there is no CPU fallback.
"""
from .kernel import packr_matmul
from .autograd import PackRMatmulFunction, PackRLinearFunction
from .layer import PackRLinear
from .layer_patcher import compress_model
from .config import PackRConfig, SchemeType
from .optim import FusedQuantizedAdam
from .cuda_adam import CUDA8BitAdam
from .velvet import VelvetController
from .offload import OffloadManager

# Legacy aliases (reference packr/__init__.py:29-34)
PHRConfig = PackRConfig
PHRLinear = PackRLinear
PHRMatmulFunction = PackRMatmulFunction
phr_matmul = packr_matmul
CV2LRTController = VelvetController

__all__ = [
    "PackRConfig", "PackRLinear", "PackRMatmulFunction", "PackRLinearFunction", "packr_matmul", "compress_model",
    "SchemeType", "FusedQuantizedAdam", "CUDA8BitAdam", "VelvetController", "OffloadManager",
    "PHRConfig", "PHRLinear", "PHRMatmulFunction", "phr_matmul", "CV2LRTController",
]
