"""GPU parity of the gated GQA attention decode layer
(li_launch_attn_layer_decode) against the oracle (oracle/li_oracle.c
lio_attn_layer_decode), through the C ABI: the hybrid stack's attention shape
(hidden 5120, 40 q heads, 8 kv heads, head_dim 128, RoPE over 64 dims, fp16
KV cache of 4096 tokens) at 1, 8 and 64 sequences, ragged positions, and
several steps with the position advancing.

Tolerances (normwise, max|got - ref| / max|ref|): 1e-3 for y when the
projections are SIMT GEMVs (up to 3 sequences), 3e-3 when they run on the
tensor cores (f16 operands in both projections, the scores' softmax between
them); the cache rows written by the step within 1e-3 (one f16 rounding) with
the SIMT projections and 2e-3 with the tensor-core in-projection (its f16
operands, then the rounding; measured up to 1.12e-3 at 24 sequences).
"""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import assert_close, elementwise_rel_err, max_rel_err, rng

pytestmark = pytest.mark.gpu


def T(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _layer(cuda, w):
    from leaninfer_b200 import ops
    return ops.AttnLayerDecode(
        hidden=w["hidden"], n_q_heads=w["n_q_heads"], n_kv_heads=w["n_kv_heads"], head_dim=w["head_dim"],
        rope_dim=w["rope_dim"], rope_theta=w["rope_theta"], w_in=T(w["w_in"], cuda), w_out=T(w["w_out"], cuda),
        in_norm_w=T(w["in_norm_w"], cuda), q_norm_w=T(w["q_norm_w"], cuda), k_norm_w=T(w["k_norm_w"], cuda),
        w_in_type=w["wtype"], w_out_type=w["wtype"])


def _f16(u16):
    return np.asarray(u16).view(np.float16).astype(np.float32)


def _check_step(cuda, oracle_mod, layer, L, keep, x, kc, vc, kc_d, vc_d, pos, tol_y, what):
    import torch
    n = x.shape[0]
    y = torch.empty(n, L.hidden, device=cuda)
    kg0 = kc_d.cpu().numpy().view(np.uint16)
    vg0 = vc_d.cpu().numpy().view(np.uint16)
    layer.step(T(x, cuda), y, kc_d, vc_d, T(pos, cuda))
    torch.cuda.synchronize()
    y_ref = oracle_mod.attn_layer_decode(L, keep, x, kc, vc, pos)
    got = y.cpu().numpy()
    print(json.dumps({"case": what, "normwise": max_rel_err(got, y_ref),
                      "elementwise_above_1e-3_max": elementwise_rel_err(got, y_ref)}))
    assert_close(got, y_ref, tol_y, f"{what}: y")
    # the rows the step wrote (against the oracle's), and that no other row of
    # the device caches changed
    kg = kc_d.cpu().numpy().view(np.uint16)
    vg = vc_d.cpu().numpy().view(np.uint16)
    tol_row = 1e-3 if n <= 2 else 2e-3
    for s in range(n):
        assert_close(_f16(kg[s, pos[s]]), _f16(kc[s, pos[s]]), tol_row, f"{what}: k row s={s}")
        assert_close(_f16(vg[s, pos[s]]), _f16(vc[s, pos[s]]), tol_row, f"{what}: v row s={s}")
    mask = np.ones(kc.shape[:2], bool)
    mask[np.arange(n), pos] = False
    assert np.array_equal(kg[mask], kg0[mask]) and np.array_equal(vg[mask], vg0[mask])


@pytest.mark.parametrize("B,wtype", [(1, 12), (8, 12), (64, 12), (2, 8), (5, 8)])
def test_attn_layer_decode_ctx4096(cuda, oracle_mod, B, wtype):
    """Every sequence attends over a full 4096-token cache (the new token at
    slot 4095) at the hybrid stack's attention shape."""
    import torch
    from leaninfer_b200 import synth
    r = rng(6000 + B + wtype)
    w = synth.attn_layer(r, hidden=5120, n_q_heads=40, n_kv_heads=8, wtype=wtype)
    layer = _layer(cuda, w)
    L, keep = oracle_mod.make_attn_layer(w)
    inp = synth.attn_inputs(r, B, w, 4096)
    kc_d = T(inp["k_cache"], cuda).view(torch.float16)
    vc_d = T(inp["v_cache"], cuda).view(torch.float16)
    tol = 1e-3 if B <= 2 else 3e-3
    _check_step(cuda, oracle_mod, layer, L, keep, inp["x"], inp["k_cache"], inp["v_cache"], kc_d, vc_d,
                inp["pos"], tol, f"attn B={B} w{wtype} ctx4096")
    from leaninfer_b200 import ops
    assert ops.device_status() == 0


@pytest.mark.parametrize("B,G,max_ctx", [(3, 5, 700), (6, 4, 700), (4, 1, 700), (24, 5, 6000), (40, 8, 4000)])
def test_attn_layer_ragged_positions_and_steps(cuda, oracle_mod, B, G, max_ctx):
    """Ragged contexts (a sequence at its first token, others mid-cache) and
    three steps with every position advancing by one, at hidden 1024 with
    Hq/Hkv = G; rope over 32 dims. The first three cases split the context
    into 64-token chunks (the CUDA-core attention kernel); the last two into
    256-token chunks (the tensor-core kernel: 128-token tiles, the last tile
    of each sequence partly past its position, chunks past it skipped)."""
    import torch
    from leaninfer_b200 import synth
    r = rng(6100 + 10 * B + G)
    Hkv = 2
    w = synth.attn_layer(r, hidden=1024, n_q_heads=Hkv * G, n_kv_heads=Hkv, rope_dim=32, wtype=12)
    layer = _layer(cuda, w)
    L, keep = oracle_mod.make_attn_layer(w)
    pos = np.array([0] + list(r.integers(1, max_ctx - 3, size=B - 1)), np.int32)
    inp = synth.attn_inputs(r, B, w, max_ctx, pos)
    kc, vc = inp["k_cache"], inp["v_cache"]
    kc_d = T(kc, cuda).view(torch.float16)
    vc_d = T(vc, cuda).view(torch.float16)
    tol = 1e-3 if B <= 2 else 3e-3
    for step in range(3):
        x = r.standard_normal((B, 1024)).astype(np.float32)
        p = pos + step
        _check_step(cuda, oracle_mod, layer, L, keep, x, kc, vc, kc_d, vc_d, p, tol, f"attn ragged step {step}")


@pytest.mark.parametrize("B,max_ctx", [(3, 300), (24, 6000)])
def test_attn_position_outside_the_cache_raises_the_device_flag(cuda, oracle_mod, B, max_ctx):
    """A position at max_ctx (one past the last slot) and one at -1: the
    kernels' bounds checks write and read no cache row for those sequences,
    li_device_status() reports LI_ERR_BAD_ARG, the other sequences' outputs
    are the oracle's and their cache rows are written. 3 sequences (64-token
    chunks, the CUDA-core attention kernel) and 24 (256-token chunks, the
    tensor-core kernel)."""
    import torch
    from leaninfer_b200 import ops, synth
    r = rng(6300 + B)
    w = synth.attn_layer(r, hidden=1024, n_q_heads=8, n_kv_heads=2, rope_dim=32, wtype=12)
    layer = _layer(cuda, w)
    L, keep = oracle_mod.make_attn_layer(w)
    pos = np.array([max_ctx // 2, max_ctx] + [max_ctx // 3] * (B - 3) + [-1], np.int32)
    inp = synth.attn_inputs(r, B, w, max_ctx, np.clip(pos, 0, max_ctx - 1))
    kc, vc = inp["k_cache"], inp["v_cache"]
    kc_d, vc_d = T(kc, cuda).view(torch.float16), T(vc, cuda).view(torch.float16)
    x = r.standard_normal((B, 1024)).astype(np.float32)
    y = torch.empty(B, 1024, device=cuda)
    layer.step(T(x, cuda), y, kc_d, vc_d, T(pos, cuda))
    assert ops.device_status() == 2001                       # LI_ERR_BAD_ARG
    got = y.cpu().numpy()
    assert np.all(np.isfinite(got))
    bad = [1, B - 1]
    kg, vg = kc_d.cpu().numpy().view(np.uint16), vc_d.cpu().numpy().view(np.uint16)
    for s in bad:                                            # nothing written for the bad positions
        assert np.array_equal(kg[s], kc[s]) and np.array_equal(vg[s], vc[s])
    good = [s for s in range(B) if s not in bad]
    y_ref = oracle_mod.attn_layer_decode(L, keep, x[good], kc[good].copy(), vc[good].copy(), pos[good])
    assert_close(got[good], y_ref, 1e-3 if B <= 2 else 3e-3, "valid sequences")
    assert ops.device_status() == 0
