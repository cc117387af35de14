"""hayai_b200 -- B200-native (sm_100a) quantized-FFN backend for Hayai.

The compute lives in ``lib/libhayai_cuda.so`` (hand-written CUDA, C ABI declared in
``include/hayai_cuda.h``); this package is the host-side mirror of the reference's
matmul / FFN op API on top of it.
"""
from .engine import (BF16, BLOCK, F16, F32, IQ2_S, IQ2_XS, IQ2_XXS, IQ3_S, IQ3_XXS, IQ4_NL, IQ4_XS, Q2_K,  # noqa: F401
                     Q3_K, Q4_0, Q4_1, Q4_K, Q5_0, Q5_1, Q5_K, Q6_K, Q8_0, Q8_1, Q8_K, TYPE_LABELS, BoundStack, CudaEngine,
                     CudaError,
                     PendingGemv, QuantMatrix, ResidentWeights, device_count, row_bytes)
from .orchestrator import EngineOrchestrator

__all__ = ["BoundStack", "CudaEngine", "CudaError", "EngineOrchestrator", "PendingGemv", "QuantMatrix", "ResidentWeights",
           "device_count", "row_bytes", "F32", "Q8_0", "Q4_K", "Q6_K", "IQ2_XXS", "IQ2_XS", "IQ2_S", "IQ3_XXS",
           "IQ3_S", "Q4_0", "Q4_1", "Q5_0", "Q5_1", "Q2_K", "Q3_K", "Q5_K", "IQ4_NL", "IQ4_XS", "F16", "BF16",
           "Q8_1", "Q8_K", "BLOCK",
           "TYPE_LABELS"]
