"""LeanInfer fused-kernel path, B200 (sm_100a) implementation.

The product is the C-ABI library ``libleaninfer_cuda.so`` (declared in
include/leaninfer-cuda.h); ``ops`` wraps it for torch tensors, ``synth``
builds seeded ggml-block inputs, ``build`` compiles it.
"""
from ._lib import LeanInferError, load  # noqa: F401

__all__ = ["LeanInferError", "load"]
