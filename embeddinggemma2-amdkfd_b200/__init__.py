"""B200-native executor for the EmbeddingGemma 2 packed-wave text graph.

Drop-in for p3psi-boo/EmbeddingGemma2-AMDKFD's executor C ABI
(src/gemma2_kfd.h) and operator surface (kernels/abi.h), implemented as
hand-written sm_100a CUDA in libeg2_b200.so.  The directory name is not a
Python identifier; import it with
``importlib.import_module("embeddinggemma2-amdkfd_b200")``.
"""
from . import _lib, synthetic  # noqa: F401
from .executor import (EMBED_DIM, MAX_TOKENS, WIDE_MAX_TOKENS, ExecutorError, GGUFModel,  # noqa: F401
                       Gemma2Executor, normalize_prefix, validate, validate_rows)

__all__ = ["GGUFModel", "Gemma2Executor", "ExecutorError", "normalize_prefix", "validate", "validate_rows",
           "EMBED_DIM", "MAX_TOKENS", "WIDE_MAX_TOKENS"]
