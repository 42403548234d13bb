"""anelm_b200: B200 (sm_100a) attention core for Qwen3.5-style hybrid models.

Replaces the CPU attention core ANE-LM runs between its projection chunks
(core/cpu_ops.cpp, models/llm/qwen3_5.cpp:849-1002, scripts/serve_hybrid.py:85-132)
with hand-written CUDA kernels behind the C ABI of include/anelm_b200.h.
"""
from ._lib import (AnelmError, BF16, DELTA_CPUOPS, DELTA_HF, ERR_CAPACITY, ERR_CUDA, ERR_INVALID_ARG,  # noqa: F401
                   ERR_NOMEM, ERR_STATE, ERR_TIMEOUT, ERR_UNSUPPORTED, F16, F32, KV_LINEAR, KV_RING,
                   LAYER_FULL_ATTN, LAYER_LINEAR_ATTN, LIB_PATH, ROPE_HALF, ROPE_INTERLEAVED, lib)


def __getattr__(name):
    # torch-dependent pieces load lazily so the ctypes layer imports without torch
    if name in ("Context", "Plan"):
        from . import core
        return getattr(core, name)
    if name == "CudaAttention":
        from .serve_hybrid import CudaAttention
        return CudaAttention
    raise AttributeError(name)
