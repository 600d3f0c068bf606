"""B200-native (sm_100a) backend for the mini-MLA engine's online GRPO step.

The compute path is ``libmm_cuda.so`` (hand-written CUDA behind the C ABI of
include/mm_cuda.h); this package is its host-side mirror of the reference's Execution
interface (``engine``) plus the model configuration (``config``).
"""
from .config import MLA36M, TINY, AdamWConfig, ModelConfig  # noqa: F401
from .engine import (CudaExecution, EngineError, cosine_learning_rate, init_params,  # noqa: F401
                     lib, make_execution, parameter_count)

__all__ = ["ModelConfig", "AdamWConfig", "TINY", "MLA36M", "CudaExecution", "EngineError",
           "make_execution", "init_params", "parameter_count", "cosine_learning_rate", "lib"]
