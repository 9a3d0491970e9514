"""Host-side mirror of the hybrid stack decode entry (li_launch_stack_decode).

A stack is a list of layers, each a mixer (Gated DeltaNet or gated GQA
attention) followed by a SwiGLU FFN; one step runs every layer on the
residual stream x in place (x += mixer(x); x += ffn(x)). The device tensors
(weights, recurrent states, conv states, KV caches) are the caller's; this
module only builds the C descriptors that point at them and calls the entry
on torch's current stream.

The weights can come from numpy (tests: random-code blocks from synth) or be
drawn on the device (benchmark: ``random_q4_k_device``), in the raw ggml
block layout either way.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from ._lib import (LI_LAYER_ATTN, LI_LAYER_DELTANET, LI_WTYPE_Q4_K, AttnLayer, DeltaNetLayer, FfnWeights,
                   StackLayer, check)


def _p(t):
    if t is None:
        return None
    assert t.is_cuda and t.is_contiguous()
    return t.data_ptr()


def random_q4_k_device(n: int, k: int, device, generator=None) -> torch.Tensor:
    """[n, k/256*144] uint8 Q4_K rows drawn on the device with the synth
    distributions: fp16 d, dmin ~ U(1e-3, 1e-2), uniform scale bytes and
    nibbles."""
    nb = k // 256
    blocks = torch.randint(0, 256, (n, nb, 144), dtype=torch.uint8, device=device, generator=generator)
    dd = (torch.rand(n, nb, 2, device=device, generator=generator) * 9e-3 + 1e-3).half()
    blocks[:, :, 0:4] = dd.view(torch.uint8).view(n, nb, 4)
    return blocks.view(n, nb * 144)


class HybridStackDecode:
    """Layers: dicts with key "kind" ("deltanet" or "attn"), the mixer's
    weights and per-sequence state tensors, and "ffn" (a dict with wtype,
    hidden, n_inner, norm_w, w_gate, w_up, w_down)."""

    def __init__(self, layers: list[dict], *, n_seqs: int, max_ctx: int, tp_comm=None, tp_nranks: int = 1):
        self.layers = layers
        self.n_seqs, self.max_ctx = n_seqs, max_ctx
        self.tp_comm, self.tp_nranks = tp_comm, tp_nranks
        self._keep = []
        arr = (StackLayer * len(layers))()
        for i, l in enumerate(layers):
            d = arr[i]
            if l["kind"] == "deltanet":
                dl = DeltaNetLayer(
                    hidden=l["hidden"], n_k_heads=l["n_k_heads"], n_v_heads=l["n_v_heads"], head_dim=l["head_dim"],
                    conv_kernel=4, repeat_type=0, w_in_type=l["wtype"], w_out_type=l["wtype"],
                    in_norm_eps=l.get("eps", 1e-6), norm_eps=l.get("eps", 1e-6), l2_eps=1e-6,
                    in_norm_w=_p(l["in_norm_w"]), w_in=_p(l["w_in"]), conv_w=_p(l["conv_w"]), a_log=_p(l["a_log"]),
                    dt_bias=_p(l["dt_bias"]), norm_w=_p(l["norm_w"]), w_out=_p(l["w_out"]))
                self._keep.append(dl)
                d.kind = LI_LAYER_DELTANET
                d.deltanet = ctypes.pointer(dl)
                d.conv_state = _p(l["conv_state"])
                d.state = _p(l["state"])
            else:
                al = AttnLayer(
                    hidden=l["hidden"], n_q_heads=l["n_q_heads"], n_kv_heads=l["n_kv_heads"], head_dim=l["head_dim"],
                    rope_dim=l["rope_dim"], w_in_type=l["wtype"], w_out_type=l["wtype"], rope_theta=l["rope_theta"],
                    in_norm_eps=l.get("eps", 1e-6), qk_norm_eps=l.get("eps", 1e-6), in_norm_w=_p(l["in_norm_w"]),
                    w_in=_p(l["w_in"]), q_norm_w=_p(l.get("q_norm_w")), k_norm_w=_p(l.get("k_norm_w")),
                    w_out=_p(l["w_out"]))
                self._keep.append(al)
                d.kind = LI_LAYER_ATTN
                d.attn = ctypes.pointer(al)
                d.k_cache = _p(l["k_cache"])
                d.v_cache = _p(l["v_cache"])
            f = l["ffn"]
            d.ffn = FfnWeights(wtype=f.get("wtype", LI_WTYPE_Q4_K), hidden=f["hidden"], n_inner=f["n_inner"],
                               eps=f.get("eps", 1e-6), norm_w=_p(f["norm_w"]), w_gate=_p(f["w_gate"]),
                               w_up=_p(f["w_up"]), w_down=_p(f["w_down"]))
        self.desc = arr
        lib = _lib.load()
        need = int(lib.li_stack_workspace_size(arr, len(layers), n_seqs, max_ctx, tp_nranks))
        if need == 0:
            raise ValueError("li_stack_workspace_size rejected the stack description")
        self.workspace = torch.empty(need, dtype=torch.uint8, device=layers[0]["w_in"].device)

    def step(self, x: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """One token per sequence through every layer; x updated in place."""
        assert x.shape[0] == self.n_seqs and pos.dtype == torch.int32
        check(_lib.load().li_launch_stack_decode(
            self.desc, len(self.layers), _p(x), _p(pos), self.n_seqs, self.max_ctx,
            ctypes.c_void_p(self.tp_comm) if self.tp_comm else None, self.tp_nranks, _p(self.workspace),
            self.workspace.numel(), torch.cuda.current_stream().cuda_stream), "li_launch_stack_decode")
        return x
