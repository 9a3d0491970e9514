"""ctypes binding of ``libleaninfer_cuda.so`` (the C ABI in include/leaninfer-cuda.h).

The library is the product: when it is missing this module raises instead of
falling back to anything else.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_float, c_int, c_int64, c_size_t, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libleaninfer_cuda.so")

LI_WTYPE_F32, LI_WTYPE_F16, LI_WTYPE_Q8_0, LI_WTYPE_Q4_K = 0, 1, 8, 12

STATUS_NAMES = {
    0: "LI_OK",
    2001: "LI_ERR_BAD_ARG",
    2002: "LI_ERR_BAD_SHAPE",
    2003: "LI_ERR_UNSUPPORTED",
    2004: "LI_ERR_WORKSPACE",
    2005: "LI_ERR_MISALIGNED",
    2006: "LI_ERR_TIMEOUT",
    2007: "LI_ERR_NO_CUDA",
    2008: "LI_ERR_SCRATCH_LIMIT",
    2009: "LI_ERR_NCCL",
}


class LeanInferError(RuntimeError):
    def __init__(self, code: int, what: str = ""):
        self.code = code
        name = STATUS_NAMES.get(code, f"cudaError {code}")
        super().__init__(f"{what}: {name} ({code})" if what else f"{name} ({code})")


class DeltaNetLayer(ctypes.Structure):
    """Mirror of ``li_deltanet_layer``."""

    _fields_ = [
        ("hidden", c_int), ("n_k_heads", c_int), ("n_v_heads", c_int),
        ("head_dim", c_int), ("conv_kernel", c_int), ("repeat_type", c_int),
        ("w_in_type", c_int), ("w_out_type", c_int),
        ("in_norm_eps", c_float), ("norm_eps", c_float), ("l2_eps", c_float),
        ("in_norm_w", c_void_p), ("w_in", c_void_p), ("conv_w", c_void_p),
        ("a_log", c_void_p), ("dt_bias", c_void_p), ("norm_w", c_void_p),
        ("w_out", c_void_p),
    ]


class AttnLayer(ctypes.Structure):
    """Mirror of ``li_attn_layer``."""

    _fields_ = [
        ("hidden", c_int), ("n_q_heads", c_int), ("n_kv_heads", c_int), ("head_dim", c_int),
        ("rope_dim", c_int), ("w_in_type", c_int), ("w_out_type", c_int),
        ("rope_theta", c_float), ("in_norm_eps", c_float), ("qk_norm_eps", c_float),
        ("in_norm_w", c_void_p), ("w_in", c_void_p), ("q_norm_w", c_void_p), ("k_norm_w", c_void_p),
        ("w_out", c_void_p),
    ]


class FfnWeights(ctypes.Structure):
    """Mirror of ``li_ffn_weights``."""

    _fields_ = [
        ("wtype", c_int), ("hidden", c_int), ("n_inner", c_int), ("eps", c_float),
        ("norm_w", c_void_p), ("w_gate", c_void_p), ("w_up", c_void_p), ("w_down", c_void_p),
    ]


class StackLayer(ctypes.Structure):
    """Mirror of ``li_stack_layer``."""

    _fields_ = [
        ("kind", c_int), ("deltanet", POINTER(DeltaNetLayer)), ("conv_state", c_void_p), ("state", c_void_p),
        ("attn", POINTER(AttnLayer)), ("k_cache", c_void_p), ("v_cache", c_void_p), ("ffn", FfnWeights),
    ]


LI_LAYER_DELTANET, LI_LAYER_ATTN = 1, 2


class GgmlTensor(ctypes.Structure):
    """Mirror of ``li_ggml_tensor`` (include/leaninfer-ggml.h)."""


GgmlTensor._fields_ = [
    ("type", ctypes.c_int32), ("ne", c_int64 * 4), ("nb", c_size_t * 4), ("op", ctypes.c_int32),
    ("op_params", ctypes.c_int32 * 16), ("src", POINTER(GgmlTensor) * 10), ("data", c_void_p),
]


# name -> (restype, argtypes)
_SIGS = {
    # reference entries (void)
    "li_launch_fused_rms_norm_matmul_f32": (None, [c_void_p] * 4 + [c_int, c_int, c_float, c_void_p]),
    "li_launch_fused_rms_norm_swiglu_f32": (None, [c_void_p] * 5 + [c_int, c_int, c_float, c_void_p]),
    "li_launch_fused_rms_norm_swiglu_f16": (None, [c_void_p] * 5 + [c_int, c_int, c_float, c_void_p]),
    "li_launch_fused_rms_norm_silu_gate_f32": (None, [c_void_p] * 4 + [c_int, c_int, c_float, c_void_p]),
    "li_launch_fused_deltanet_recurrent_out_f32": (
        None, [c_void_p] * 9 + [c_int64, c_int64, c_int64, c_int64, c_int, c_int64, c_int64,
                                c_size_t, c_size_t, c_size_t, c_void_p]),
    "li_launch_fused_rms_norm_qkv_f32": (
        None, [c_void_p, c_void_p, POINTER(c_void_p), POINTER(c_void_p), c_int, c_int, c_float, c_void_p]),
    "li_get_last_error": (c_int, []),
    # additive entries (int status)
    "li_device_status": (c_int, []),
    "li_row_bytes": (c_size_t, [c_int, c_int64]),
    "li_selftest_bounded_wait": (c_int, [c_int, c_void_p, c_void_p]),
    "li_launch_add_f32": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "li_launch_dequantize": (c_int, [c_int, c_void_p, c_void_p, c_int64, c_void_p]),
    "li_launch_rms_norm_matmul_q": (
        c_int, [c_int] + [c_void_p] * 4 + [c_int, c_int, c_int, c_float, c_void_p]),
    "li_launch_fused_rms_norm_qkv_q": (
        c_int, [c_int] + [c_void_p] * 8 + [c_int] * 5 + [c_float, c_void_p]),
    "li_launch_fused_rms_norm_swiglu_q": (
        c_int, [c_int] + [c_void_p] * 5 + [c_int, c_int, c_int, c_float, c_void_p]),
    "li_fused_ffn_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "li_launch_fused_ffn_q": (
        c_int, [c_int] + [c_void_p] * 6 + [c_int, c_int, c_int, c_float, c_void_p, c_size_t, c_void_p]),
    "li_launch_deltanet_recurrent_f32": (
        c_int, [c_void_p] * 8 + [c_int64, c_int64, c_int64, c_int64, c_int, c_int64,
                                 c_size_t, c_size_t, c_size_t, c_void_p]),
    "li_deltanet_layer_workspace_size": (c_size_t, [POINTER(DeltaNetLayer), c_int]),
    "li_deltanet_chunk_prefill_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "li_launch_deltanet_chunk_prefill_bf16": (c_int, [c_void_p] * 7 + [c_int] * 4 + [c_float, c_void_p, c_size_t,
                                                                                     c_void_p]),
    "li_launch_gated_rmsnorm_bf16": (c_int, [c_void_p] * 4 + [c_int, c_int64, c_float, c_void_p]),
    "li_launch_gemm_bf16_f32": (c_int, [c_void_p] * 3 + [c_int] * 3 + [c_void_p]),
    "li_launch_deltanet_layer_decode": (
        c_int, [POINTER(DeltaNetLayer), c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                c_void_p, c_size_t, c_void_p]),
    "li_launch_deltanet_layer_decode_f16state": (
        c_int, [POINTER(DeltaNetLayer), c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                c_void_p, c_size_t, c_void_p]),
    "li_launch_deltanet_layer_decode_noalloc": (
        c_int, [POINTER(DeltaNetLayer), c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    "li_attn_layer_workspace_size": (c_size_t, [POINTER(AttnLayer), c_int, c_int]),
    "li_launch_attn_layer_decode": (
        c_int, [POINTER(AttnLayer)] + [c_void_p] * 5 + [c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "li_nccl_available": (c_int, []),
    "li_nccl_get_unique_id": (c_int, [c_void_p]),
    "li_nccl_comm_init_rank": (c_int, [POINTER(c_void_p), c_int, c_void_p, c_int]),
    "li_nccl_comm_destroy": (c_int, [c_void_p]),
    "li_ffn_tp_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int]),
    "li_launch_ffn_q_tp": (
        c_int, [c_int] + [c_void_p] * 6 + [c_int, c_int, c_int, c_float, c_void_p, c_int, c_void_p, c_size_t,
                                           c_void_p]),
    "li_stack_workspace_size": (c_size_t, [POINTER(StackLayer), c_int, c_int, c_int, c_int]),
    "li_launch_stack_decode": (
        c_int, [POINTER(StackLayer), c_int, c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_void_p, c_size_t,
                c_void_p]),
    # ggml-style node dispatch (include/leaninfer-ggml.h)
    "li_ggml_workspace_size": (c_size_t, [c_void_p]),
    "li_ggml_compute_forward": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
}

_lib = None


def load(path: Path | None = None) -> ctypes.CDLL:
    """Load the CUDA library once. Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise LeanInferError(2007, f"{p} is missing; run `python -m leaninfer_b200.build` "
                                   "(the CUDA library is required, there is no fallback)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def exported_names() -> list[str]:
    return list(_SIGS)


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise LeanInferError(rc, what)
