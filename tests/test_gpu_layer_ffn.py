"""GPU parity of the DeltaNet + FFN decode layer at the benchmarked shapes
(bench.py --workload layerffn): the Gated DeltaNet layer with hidden 4096,
16 k-heads, 32 v-heads, head_dim 128, followed by the SwiGLU FFN 4096 ->
12288 -> 4096, Q4_K, a residual add after each, one li_launch_stack_decode
call per step. 1 sequence (SIMT GEMVs), 8 (X-stationary tensor-core GEMMs)
and 64 (one-tile tensor-core GEMMs, the benchmarked batch), two steps.

Each step is checked on the GPU's own intermediates, every part against the
oracle at its own tolerance:
- the DeltaNet layer's output y for the step's x and pre-step states (the
  same entry run alone on copies of them; the stack calls it with the same
  arguments) against the oracle's layer: 1e-3 normwise with fp32 operands (1
  sequence), 2e-3 with the tensor cores' f16 operands;
- the stack's residual stream after the step against x + y + oracle FFN(x +
  y), y the GPU's: 1e-3;
- the recurrent and conv states after the step against the oracle's layer
  step from the same pre-step states: 1e-3.
Comparing the stack with the oracle's whole composition instead measures the
conditioning of these random-weight FFNs: at one sequence the GPU's y
differs from the oracle's by 6e-5 (normwise), and that difference in the
FFN's input moves the oracle FFN's own output by 4.2e-3. Each step also
reports the elementwise relative error over the elements above 1e-3 of the
largest magnitude."""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import assert_close, elementwise_rel_err, max_rel_err, rng

pytestmark = pytest.mark.gpu
HIDDEN, HK, HV, D, FFN = 4096, 16, 32, 128, 12288


def T(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def report(case, got, ref):
    nw, ew = max_rel_err(got, ref), elementwise_rel_err(got, ref)
    print(json.dumps({"case": case, "normwise": nw, "elementwise_above_1e-3_max": ew}))


@pytest.mark.parametrize("B", [1, 8, 64])
def test_deltanet_ffn_layer_two_steps(cuda, oracle_mod, B):
    import torch
    from leaninfer_b200 import ops, synth
    from leaninfer_b200.stack import HybridStackDecode
    r = rng(9100 + B)
    w = synth.deltanet_layer(r, hidden=HIDDEN, n_k_heads=HK, n_v_heads=HV, head_dim=D, wtype=synth.Q4_K)
    w["in_norm_w"] = (r.uniform(0.5, 1.5, HIDDEN) / 128.0).astype(np.float32)
    inp = synth.deltanet_inputs(r, B, w)
    ffn = dict(wtype=synth.Q4_K, hidden=HIDDEN, n_inner=FFN,
               norm_w=(r.uniform(0.5, 1.5, HIDDEN) / 128.0).astype(np.float32),
               w_gate=synth.random_q4_k(r, FFN, HIDDEN), w_up=synth.random_q4_k(r, FFN, HIDDEN),
               w_down=synth.random_q4_k(r, HIDDEN, FFN))
    d = {k: (T(v, cuda) if isinstance(v, np.ndarray) else v) for k, v in w.items()}
    d["kind"] = "deltanet"
    d["conv_state"], d["state"] = T(inp["conv_state"], cuda), T(inp["state"], cuda)
    d["ffn"] = {k: (T(v, cuda) if isinstance(v, np.ndarray) else v) for k, v in ffn.items()}
    stack = HybridStackDecode([d], n_seqs=B, max_ctx=1)
    alone = ops.DeltaNetLayerDecode(hidden=HIDDEN, n_k_heads=HK, n_v_heads=HV, head_dim=D, w_in=d["w_in"],
                                    conv_w=d["conv_w"], a_log=d["a_log"], dt_bias=d["dt_bias"],
                                    norm_w=d["norm_w"], w_out=d["w_out"], in_norm_w=d["in_norm_w"])
    ws = torch.empty(alone.workspace_bytes(B), device=cuda, dtype=torch.uint8)
    pos = torch.zeros(B, dtype=torch.int32, device=cuda)
    L, keep = oracle_mod.make_layer(w, in_norm_w=w["in_norm_w"])
    tol_y = 1e-3 if B == 1 else 2e-3
    xd = T(inp["x"], cuda)
    for step in range(2):
        x = xd.cpu().numpy()
        cs, st = d["conv_state"].cpu().numpy(), d["state"].cpu().numpy()
        # the layer alone on copies of the pre-step states
        yd = torch.empty(B, HIDDEN, device=cuda)
        alone.step(xd.clone(), yd, T(cs, cuda), T(st, cuda), workspace=ws)
        stack.step(xd, pos)
        torch.cuda.synchronize()
        y = yd.cpu().numpy()
        y_ref = oracle_mod.deltanet_layer_decode(L, keep, x, cs, st)      # cs, st -> post-step oracle states
        report(f"layer y B={B} step {step}", y, y_ref)
        assert_close(y, y_ref, tol_y, f"layer output B={B} step {step}")
        x1 = (x + y).astype(np.float32)
        x2 = (x1 + oracle_mod.ffn(ffn["wtype"], x1, ffn["norm_w"], ffn["w_gate"], ffn["w_up"], ffn["w_down"],
                                  FFN)).astype(np.float32)
        got = xd.cpu().numpy()
        report(f"residual after ffn B={B} step {step}", got, x2)
        assert_close(got, x2, 1e-3, f"residual stream B={B} step {step}")
        assert_close(d["state"].cpu().numpy(), st, 1e-3, f"recurrent state B={B} step {step}")
        assert_close(d["conv_state"].cpu().numpy(), cs, 1e-3, f"conv state B={B} step {step}")
    assert ops.device_status() == 0
