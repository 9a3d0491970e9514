"""GPU parity of the hybrid stack decode entry (li_launch_stack_decode)
against the oracle's layer-by-layer composition: a block of three Gated
DeltaNet layers and one gated attention layer, each followed by a SwiGLU
FFN, residual adds after every mixer and FFN, two steps with the attention
position advancing. Hidden 1024 (DeltaNet 4 k / 8 v heads, attention 8 q / 2
kv heads, FFN 1024 -> 2816, Q4_K), at 3, 8 and 40 sequences (SIMT GEMVs,
X-stationary and one-tile tensor-core projections).

Tolerances, normwise on the residual stream after each step: 2e-3 with the
SIMT projections (3 sequences, fp32 operands), 1e-2 with the tensor-core
projections (f16 operands, about 4e-4 per projection): eight sub-layers
compose, and the DeltaNet gates and the SwiGLU amplify an operand error on
some rows (the per-entry tests hold each sub-layer to its own tolerance; one
DeltaNet layer + FFN already measures up to 1.2e-3 on random inputs here). A
wiring fault (a wrong buffer, a missing residual add) gives errors of order
one. Recurrent states: the first layer's within 2e-3; the later layers'
within 2e-3 on the SIMT path and 5e-2 on the tensor-core path, where their
inputs already differ by the residual stream's error."""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import assert_close, max_rel_err, rng

pytestmark = pytest.mark.gpu


def T(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _build(r, B, max_ctx):
    from leaninfer_b200 import synth
    hidden, N = 1024, 2816
    layers = []
    for kind in ("deltanet", "deltanet", "deltanet", "attn"):
        if kind == "deltanet":
            w = synth.deltanet_layer(r, hidden=hidden, n_k_heads=4, n_v_heads=8, wtype=synth.Q4_K)
            w["in_norm_w"] = (r.uniform(0.5, 1.5, hidden) / 128.0).astype(np.float32)
            st = dict(conv_state=r.normal(0, 0.1, (B, 2 * 4 * 128 + 8 * 128, 3)).astype(np.float32),
                      state=r.normal(0, 0.02, (B, 8, 128, 128)).astype(np.float32))
        else:
            w = synth.attn_layer(r, hidden=hidden, n_q_heads=8, n_kv_heads=2, rope_dim=32, wtype=synth.Q4_K)
            a = synth.attn_inputs(r, B, w, max_ctx, pos=np.full(B, max_ctx - 2, np.int32))
            st = dict(k_cache=a["k_cache"], v_cache=a["v_cache"])
        ffn = dict(wtype=synth.Q4_K, hidden=hidden, n_inner=N,
                   norm_w=(r.uniform(0.5, 1.5, hidden) / 128.0).astype(np.float32),
                   w_gate=synth.random_q4_k(r, N, hidden), w_up=synth.random_q4_k(r, N, hidden),
                   w_down=synth.random_q4_k(r, hidden, N))
        layers.append(dict(kind=kind, w=w, st=st, ffn=ffn))
    return layers


def _oracle_step(oracle_mod, layers, x, pos):
    for l in layers:
        if l["kind"] == "deltanet":
            L, keep = oracle_mod.make_layer(l["w"], in_norm_w=l["w"]["in_norm_w"])
            t = oracle_mod.deltanet_layer_decode(L, keep, x, l["st"]["conv_state"], l["st"]["state"])
        else:
            L, keep = oracle_mod.make_attn_layer(l["w"])
            t = oracle_mod.attn_layer_decode(L, keep, x, l["st"]["k_cache"], l["st"]["v_cache"], pos)
        x = (x + t).astype(np.float32)
        f = l["ffn"]
        t = oracle_mod.ffn(f["wtype"], x, f["norm_w"], f["w_gate"], f["w_up"], f["w_down"], f["n_inner"])
        x = (x + t).astype(np.float32)
    return x


@pytest.mark.parametrize("B", [3, 8, 40])
def test_stack_block_two_steps(cuda, oracle_mod, B):
    import torch
    from leaninfer_b200.stack import HybridStackDecode
    r = rng(7700 + B)
    max_ctx = 300
    layers = _build(r, B, max_ctx)
    dev_layers = []
    for l in layers:
        d = {k: (T(v, cuda) if isinstance(v, np.ndarray) else v) for k, v in l["w"].items()}
        d["kind"] = l["kind"]
        for k, v in l["st"].items():
            d[k] = T(v, cuda) if k != "k_cache" and k != "v_cache" else T(v, cuda).view(torch.float16)
        d["ffn"] = {k: (T(v, cuda) if isinstance(v, np.ndarray) else v) for k, v in l["ffn"].items()}
        dev_layers.append(d)
    stack = HybridStackDecode(dev_layers, n_seqs=B, max_ctx=max_ctx)
    x = (r.standard_normal((B, 1024))).astype(np.float32)
    xd = T(x, cuda)
    for step in range(2):
        pos = np.full(B, max_ctx - 2 + step, np.int32)
        stack.step(xd, T(pos, cuda))
        torch.cuda.synchronize()
        x = _oracle_step(oracle_mod, layers, x, pos)
        got = xd.cpu().numpy()
        print(json.dumps({"case": f"stack B={B} step {step}", "normwise": max_rel_err(got, x)}))
        assert_close(got, x, 2e-3 if B < 4 else 1e-2, f"residual stream B={B} step {step}")
    # the first layer's state grows from the same x on both sides; the later
    # layers' inputs already carry the residual stream's difference (up to
    # 1e-2 on the tensor-core path), which their state updates inherit
    for i, (l, d) in enumerate(zip(layers, dev_layers)):
        if l["kind"] == "deltanet":
            tol = 2e-3 if (i == 0 or B < 4) else 5e-2
            assert_close(d["state"].cpu().numpy(), l["st"]["state"], tol, f"state of layer {i}, B={B}")
    from leaninfer_b200 import ops
    assert ops.device_status() == 0
