"""ggml-style node descriptors over torch tensors, for the node dispatch of
include/leaninfer-ggml.h (li_ggml_compute_forward). Shapes follow ggml:
ne[0] is the contiguous dimension."""
from __future__ import annotations

import ctypes
import struct

import torch

from . import _lib
from ._lib import GgmlTensor

F32, F16, Q8_0, Q4_K = 0, 1, 8, 12
OP_MUL_MAT, OP_FUSED_UP_GATE, OP_FUSED_RMS_SILU_GATE, OP_DELTANET_DECODE = 1, 2, 3, 4
_BLOCK = {Q8_0: (32, 34), Q4_K: (256, 144)}


def f32_desc(t: torch.Tensor) -> GgmlTensor:
    """Descriptor of an fp32 tensor; ne is its shape reversed (innermost
    first), nb the byte strides of those dimensions."""
    assert t.dtype == torch.float32
    d = GgmlTensor()
    d.type = F32
    dims = list(reversed(t.shape)) + [1] * (4 - t.dim())
    strides = list(reversed(t.stride())) + [t.numel()] * (4 - t.dim())
    for i in range(4):
        d.ne[i] = int(dims[i])
        d.nb[i] = int(strides[i]) * 4
    d.data = t.data_ptr()
    return d


def quant_desc(w: torch.Tensor, wtype: int, k: int, n: int) -> GgmlTensor:
    """Descriptor of a [n rows, k values] matrix of raw ggml blocks."""
    blk, size = _BLOCK[wtype]
    rb = k // blk * size
    d = GgmlTensor()
    d.type = wtype
    for i, (ne, nb) in enumerate([(k, size), (n, rb), (1, rb * n), (1, rb * n)]):
        d.ne[i] = ne
        d.nb[i] = nb
    d.data = w.data_ptr()
    return d


def node(op: int, out: GgmlTensor, srcs: list, params=()) -> GgmlTensor:
    """A node: `out` becomes the destination of `op` over `srcs` (None for an
    absent source); params are ints or floats (stored as their bits)."""
    out.op = op
    for i, s in enumerate(srcs):
        out.src[i] = ctypes.pointer(s) if s is not None else ctypes.POINTER(GgmlTensor)()
    for i, p in enumerate(params):
        out.op_params[i] = p if isinstance(p, int) else struct.unpack("<i", struct.pack("<f", p))[0]
    out._keep = list(srcs)   # sources stay alive with the node
    return out


def workspace_size(nd: GgmlTensor) -> int:
    return int(_lib.load().li_ggml_workspace_size(ctypes.byref(nd)))


def compute_forward(nd: GgmlTensor, workspace: torch.Tensor | None = None) -> int:
    """Runs the node on the current stream; returns the status code."""
    ws = workspace.data_ptr() if workspace is not None else None
    nbytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    return int(_lib.load().li_ggml_compute_forward(ctypes.byref(nd), ws, nbytes,
                                                   torch.cuda.current_stream().cuda_stream))
