"""Host-side mirror of the LeanInfer fused-kernel interface on torch tensors.

Each function takes CUDA tensors, calls the matching C-ABI entry of
``libleaninfer_cuda.so`` on torch's current stream and returns the outputs.
Argument meaning follows the reference launchers (cuda/leaninfer-cuda.h,
cuda/leaninfer-fused-ffn.cu, cuda/leaninfer-fused-gate.cu,
cuda/leaninfer-fused-deltanet.cu). PyTorch supplies device memory and
streams only; all arithmetic runs in the library's kernels.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from ._lib import (LI_WTYPE_Q4_K, LI_WTYPE_Q8_0, AttnLayer, DeltaNetLayer, LeanInferError, check)

__all__ = [
    "rms_norm_matmul_f32", "rms_norm_swiglu_f32", "rms_norm_swiglu_f16", "rms_norm_qkv_f32",
    "rms_norm_silu_gate_f32", "deltanet_recurrent_out_f32", "deltanet_recurrent_f32",
    "dequantize", "rms_norm_matmul_q", "rms_norm_qkv_q", "rms_norm_swiglu_q", "ffn_q",
    "DeltaNetLayerDecode", "AttnLayerDecode", "device_status", "row_bytes", "LI_WTYPE_Q8_0", "LI_WTYPE_Q4_K",
]


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _p(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("LeanInfer kernels take CUDA tensors")
    if not t.is_contiguous():
        raise ValueError("LeanInfer kernels take contiguous tensors")
    return t.data_ptr()


def _legacy_check(what: str) -> None:
    rc = _lib.load().li_get_last_error()
    if rc:
        raise LeanInferError(rc, what)


def row_bytes(wtype: int, k: int) -> int:
    return int(_lib.load().li_row_bytes(wtype, k))


def device_status() -> int:
    """Synchronise and return the device-side status flag (0 = ok)."""
    return int(_lib.load().li_device_status())


# --------------------------------------------------------------------------
# Reference entries
# --------------------------------------------------------------------------
def rms_norm_matmul_f32(x, gamma, W, eps: float = 1e-6):
    N, K = W.shape
    dst = torch.empty(N, device=x.device, dtype=torch.float32)
    _lib.load().li_launch_fused_rms_norm_matmul_f32(_p(x), _p(gamma), _p(W), _p(dst), K, N, eps, _stream())
    _legacy_check("li_launch_fused_rms_norm_matmul_f32")
    return dst


def rms_norm_swiglu_f32(x, gamma, W_gate, W_up, eps: float = 1e-6):
    N, K = W_gate.shape
    h = torch.empty(N, device=x.device, dtype=torch.float32)
    _lib.load().li_launch_fused_rms_norm_swiglu_f32(_p(x), _p(gamma), _p(W_gate), _p(W_up), _p(h),
                                                    K, N, eps, _stream())
    _legacy_check("li_launch_fused_rms_norm_swiglu_f32")
    return h


def rms_norm_swiglu_f16(x, gamma, W_gate, W_up, eps: float = 1e-6):
    N, K = W_gate.shape
    h = torch.empty(N, device=x.device, dtype=torch.float32)
    _lib.load().li_launch_fused_rms_norm_swiglu_f16(_p(x), _p(gamma), _p(W_gate), _p(W_up), _p(h),
                                                    K, N, eps, _stream())
    _legacy_check("li_launch_fused_rms_norm_swiglu_f16")
    return h


def rms_norm_qkv_f32(x, gamma, Ws, eps: float = 1e-6, device_arrays: bool = False):
    """device_arrays: pass W_ptrs / dst_ptrs as arrays in device memory (the
    form the reference's comment prescribes) instead of host arrays."""
    N, K = Ws[0].shape
    outs = [torch.empty(N, device=x.device, dtype=torch.float32) for _ in range(3)]
    if device_arrays:
        wt = torch.tensor([_p(w) for w in Ws], dtype=torch.int64, device=x.device)
        dt = torch.tensor([_p(o) for o in outs], dtype=torch.int64, device=x.device)
        wp = ctypes.cast(ctypes.c_void_p(wt.data_ptr()), ctypes.POINTER(ctypes.c_void_p))
        dp = ctypes.cast(ctypes.c_void_p(dt.data_ptr()), ctypes.POINTER(ctypes.c_void_p))
    else:
        wp = (ctypes.c_void_p * 3)(*[_p(w) for w in Ws])
        dp = (ctypes.c_void_p * 3)(*[_p(o) for o in outs])
    _lib.load().li_launch_fused_rms_norm_qkv_f32(_p(x), _p(gamma), wp, dp, K, N, eps, _stream())
    _legacy_check("li_launch_fused_rms_norm_qkv_f32")
    if device_arrays:
        torch.cuda.current_stream().synchronize()   # the pointer arrays must outlive the launch
    return tuple(outs)


def rms_norm_silu_gate_f32(output, z, gamma, eps: float = 1e-6):
    K = output.shape[-1]
    n_rows = output.numel() // K
    dst = torch.empty_like(output)
    _lib.load().li_launch_fused_rms_norm_silu_gate_f32(_p(output), _p(z), _p(gamma), _p(dst), K, n_rows,
                                                       eps, _stream())
    _legacy_check("li_launch_fused_rms_norm_silu_gate_f32")
    return dst


def deltanet_recurrent_out_f32(q, k, v, g, beta, state_in, W_out, *, head_dim, n_tokens, n_heads,
                               gqa_ratio, repeat_type, n_seqs, hidden_dim, vnb1, vnb2, vnb3):
    """Reference-layout recurrence + projection. Returns (dst, proj_out):
    dst holds per-head outputs then the final state, as in the reference."""
    out_elems = head_dim * n_tokens * n_heads * n_seqs
    dst = torch.empty(out_elems + state_in.numel(), device=q.device, dtype=torch.float32)
    proj = torch.empty(hidden_dim * n_tokens, device=q.device, dtype=torch.float32)
    _lib.load().li_launch_fused_deltanet_recurrent_out_f32(
        _p(q), _p(k), _p(v), _p(g), _p(beta), _p(state_in), _p(W_out), _p(dst), _p(proj),
        head_dim, n_tokens, n_heads, gqa_ratio, repeat_type, n_seqs, hidden_dim, vnb1, vnb2, vnb3,
        _stream())
    _legacy_check("li_launch_fused_deltanet_recurrent_out_f32")
    return dst, proj


# --------------------------------------------------------------------------
# Additive entries
# --------------------------------------------------------------------------
def dequantize(wtype: int, blocks: torch.Tensor, n: int) -> torch.Tensor:
    out = torch.empty(n, device=blocks.device, dtype=torch.float32)
    check(_lib.load().li_launch_dequantize(wtype, _p(blocks), _p(out), n, _stream()), "li_launch_dequantize")
    return out


def rms_norm_matmul_q(wtype, x, gamma, W, N: int, eps: float = 1e-6, out=None):
    n_rows, K = x.shape
    dst = out if out is not None else torch.empty(n_rows, N, device=x.device, dtype=torch.float32)
    check(_lib.load().li_launch_rms_norm_matmul_q(wtype, _p(x), _p(gamma), _p(W), _p(dst), K, N, n_rows,
                                                  eps, _stream()), "li_launch_rms_norm_matmul_q")
    return dst


def rms_norm_qkv_q(wtype, x, gamma, Wq, Wk, Wv, Nq: int, Nk: int, Nv: int, eps: float = 1e-6):
    n_rows, K = x.shape
    q = torch.empty(n_rows, Nq, device=x.device, dtype=torch.float32)
    k = torch.empty(n_rows, Nk, device=x.device, dtype=torch.float32)
    v = torch.empty(n_rows, Nv, device=x.device, dtype=torch.float32)
    check(_lib.load().li_launch_fused_rms_norm_qkv_q(wtype, _p(x), _p(gamma), _p(Wq), _p(Wk), _p(Wv),
                                                     _p(q), _p(k), _p(v), K, Nq, Nk, Nv, n_rows, eps,
                                                     _stream()), "li_launch_fused_rms_norm_qkv_q")
    return q, k, v


def rms_norm_swiglu_q(wtype, x, gamma, Wg, Wu, N: int, eps: float = 1e-6):
    n_rows, K = x.shape
    h = torch.empty(n_rows, N, device=x.device, dtype=torch.float32)
    check(_lib.load().li_launch_fused_rms_norm_swiglu_q(wtype, _p(x), _p(gamma), _p(Wg), _p(Wu), _p(h),
                                                        K, N, n_rows, eps, _stream()),
          "li_launch_fused_rms_norm_swiglu_q")
    return h


def ffn_q(wtype, x, gamma, Wg, Wu, Wd, N: int, eps: float = 1e-6, workspace=None, out=None):
    n_rows, K = x.shape
    lib = _lib.load()
    ws_bytes = int(lib.li_fused_ffn_workspace_size(K, N, n_rows))
    if workspace is None:
        workspace = torch.empty(ws_bytes, device=x.device, dtype=torch.uint8)
    y = out if out is not None else torch.empty(n_rows, K, device=x.device, dtype=torch.float32)
    check(lib.li_launch_fused_ffn_q(wtype, _p(x), _p(gamma), _p(Wg), _p(Wu), _p(Wd), _p(y), K, N, n_rows,
                                    eps, _p(workspace), workspace.numel(), _stream()),
          "li_launch_fused_ffn_q")
    return y


def deltanet_recurrent_f32(q, k, v, g, beta, state_in, *, head_dim, n_tokens, n_heads, gqa_ratio,
                           repeat_type, n_seqs, vnb1, vnb2, vnb3, state_out=None):
    out = torch.empty(n_seqs * n_tokens * n_heads * head_dim, device=q.device, dtype=torch.float32)
    so = state_out if state_out is not None else torch.empty_like(state_in)
    check(_lib.load().li_launch_deltanet_recurrent_f32(
        _p(q), _p(k), _p(v), _p(g), _p(beta), _p(state_in), _p(out), _p(so), head_dim, n_tokens,
        n_heads, gqa_ratio, repeat_type, n_seqs, vnb1, vnb2, vnb3, _stream()),
        "li_launch_deltanet_recurrent_f32")
    return out, so


def deltanet_chunk_prefill_bf16(q, k, v, g, beta, state, scale: float, workspace=None, out=None):
    """Chunked (WY, chunk 64) gated delta rule prefill of one sequence on the
    tensor cores. q, k bf16 [T, Hk, D]; v bf16 [T, Hv, D]; g (log decay), beta
    fp32 [T, Hv]; state fp32 [Hv, D, D] updated in place. Returns o fp32
    [T, Hv, D]."""
    T, Hk, D = q.shape
    Hv = v.shape[1]
    lib = _lib.load()
    ws_bytes = int(lib.li_deltanet_chunk_prefill_workspace_size(T, Hv, D))
    if workspace is None:
        workspace = torch.empty(max(ws_bytes, 16), device=q.device, dtype=torch.uint8)
    o = out if out is not None else torch.empty(T, Hv, D, device=q.device, dtype=torch.float32)
    check(lib.li_launch_deltanet_chunk_prefill_bf16(_p(q), _p(k), _p(v), _p(g), _p(beta), _p(state), _p(o), T, Hk,
                                                    Hv, D, scale, _p(workspace), workspace.numel(), _stream()),
          "li_launch_deltanet_chunk_prefill_bf16")
    return o


def gated_rmsnorm_bf16(o, z, gamma, eps: float = 1e-6):
    """bf16(silu(z) * rmsnorm(o) * gamma) over the last dimension."""
    K = o.shape[-1]
    n = o.numel() // K
    dst = torch.empty(o.shape, device=o.device, dtype=torch.bfloat16)
    check(_lib.load().li_launch_gated_rmsnorm_bf16(_p(o), _p(z), _p(gamma), _p(dst), K, n, eps, _stream()),
          "li_launch_gated_rmsnorm_bf16")
    return dst


def gemm_bf16(A, W, out=None):
    """C (fp32) = A . W^T with A [M, K], W [N, K] bf16, on the tensor cores."""
    M, K = A.shape
    N = W.shape[0]
    C = out if out is not None else torch.empty(M, N, device=A.device, dtype=torch.float32)
    check(_lib.load().li_launch_gemm_bf16_f32(_p(A), _p(W), _p(C), M, N, K, _stream()), "li_launch_gemm_bf16_f32")
    return C


class DeltaNetLayerDecode:
    """One DeltaNet layer's device weights plus a workspace, stepping B
    sequences one token at a time through li_launch_deltanet_layer_decode."""

    def __init__(self, *, hidden, n_k_heads, n_v_heads, head_dim, w_in, conv_w, a_log, dt_bias,
                 norm_w, w_out, w_in_type=LI_WTYPE_Q4_K, w_out_type=LI_WTYPE_Q4_K, in_norm_w=None,
                 in_norm_eps=1e-6, norm_eps=1e-6, l2_eps=1e-6, repeat_type=0, conv_kernel=4):
        self.keep = [w_in, conv_w, a_log, dt_bias, norm_w, w_out, in_norm_w]
        self.L = DeltaNetLayer(
            hidden=hidden, n_k_heads=n_k_heads, n_v_heads=n_v_heads, head_dim=head_dim,
            conv_kernel=conv_kernel, repeat_type=repeat_type, w_in_type=w_in_type,
            w_out_type=w_out_type, in_norm_eps=in_norm_eps, norm_eps=norm_eps, l2_eps=l2_eps,
            in_norm_w=_p(in_norm_w), w_in=_p(w_in), conv_w=_p(conv_w), a_log=_p(a_log),
            dt_bias=_p(dt_bias), norm_w=_p(norm_w), w_out=_p(w_out))
        self.device = w_in.device
        self._ws = None

    @classmethod
    def from_gguf(cls, path, il: int, *, n_k_heads: int, n_v_heads: int, head_dim: int = 128, names=None,
                  device="cuda", **kw) -> "DeltaNetLayerDecode":
        """Layer `il` of a GGUF checkpoint (leaninfer_b200.gguf_file: the
        quantized rows are copied to the device as they are in the file)."""
        from .gguf_file import GGUFFile, deltanet_layer
        with GGUFFile(path) as g:
            w = deltanet_layer(g, il, n_k_heads=n_k_heads, n_v_heads=n_v_heads, head_dim=head_dim, names=names)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)
        return cls(hidden=w["hidden"], n_k_heads=n_k_heads, n_v_heads=n_v_heads, head_dim=head_dim,
                   w_in=t(w["w_in"]), conv_w=t(w["conv_w"]), a_log=t(w["a_log"]), dt_bias=t(w["dt_bias"]),
                   norm_w=t(w["norm_w"]), w_out=t(w["w_out"]), w_in_type=w["wtype"], w_out_type=w["wtype"], **kw)

    @property
    def conv_channels(self) -> int:
        L = self.L
        return 2 * L.n_k_heads * L.head_dim + L.n_v_heads * L.head_dim

    def workspace_bytes(self, n_seqs: int) -> int:
        return int(_lib.load().li_deltanet_layer_workspace_size(ctypes.byref(self.L), n_seqs))

    def workspace(self, n_seqs: int) -> torch.Tensor:
        need = self.workspace_bytes(n_seqs)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, device=self.device, dtype=torch.uint8)
        return self._ws

    def step(self, x, y, conv_state, state, workspace=None):
        """One decode step; a float16 `state` takes the fp16-state entry."""
        n_seqs = x.shape[0]
        ws = workspace if workspace is not None else self.workspace(n_seqs)
        name = "li_launch_deltanet_layer_decode_f16state" if state.dtype == torch.float16 else \
            "li_launch_deltanet_layer_decode"
        check(getattr(_lib.load(), name)(
            ctypes.byref(self.L), _p(x), _p(y), _p(conv_state), _p(state), n_seqs, _p(ws), ws.numel(),
            _stream()), name)
        return y


class AttnLayerDecode:
    """One gated attention layer's device weights plus a workspace, stepping
    B sequences one token at a time through li_launch_attn_layer_decode
    against caller-owned fp16 KV caches [B, max_ctx, Hkv, D]."""

    def __init__(self, *, hidden, n_q_heads, n_kv_heads, head_dim, w_in, w_out, rope_dim=64,
                 rope_theta=1e7, in_norm_w=None, q_norm_w=None, k_norm_w=None, w_in_type=LI_WTYPE_Q4_K,
                 w_out_type=LI_WTYPE_Q4_K, in_norm_eps=1e-6, qk_norm_eps=1e-6):
        self.keep = [w_in, w_out, in_norm_w, q_norm_w, k_norm_w]
        self.L = AttnLayer(
            hidden=hidden, n_q_heads=n_q_heads, n_kv_heads=n_kv_heads, head_dim=head_dim, rope_dim=rope_dim,
            w_in_type=w_in_type, w_out_type=w_out_type, rope_theta=rope_theta, in_norm_eps=in_norm_eps,
            qk_norm_eps=qk_norm_eps, in_norm_w=_p(in_norm_w), w_in=_p(w_in), q_norm_w=_p(q_norm_w),
            k_norm_w=_p(k_norm_w), w_out=_p(w_out))
        self.device = w_in.device
        self._ws = None

    def workspace_bytes(self, n_seqs: int, max_ctx: int) -> int:
        return int(_lib.load().li_attn_layer_workspace_size(ctypes.byref(self.L), n_seqs, max_ctx))

    def workspace(self, n_seqs: int, max_ctx: int) -> torch.Tensor:
        need = self.workspace_bytes(n_seqs, max_ctx)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, device=self.device, dtype=torch.uint8)
        return self._ws

    def step(self, x, y, k_cache, v_cache, pos, workspace=None):
        """One decode step: the new token of sequence s goes to slot pos[s]
        (an int32 device tensor) of the caches."""
        n_seqs, max_ctx = x.shape[0], k_cache.shape[1]
        ws = workspace if workspace is not None else self.workspace(n_seqs, max_ctx)
        check(_lib.load().li_launch_attn_layer_decode(
            ctypes.byref(self.L), _p(x), _p(y), _p(k_cache), _p(v_cache), _p(pos), n_seqs, max_ctx, _p(ws),
            ws.numel(), _stream()), "li_launch_attn_layer_decode")
        return y
