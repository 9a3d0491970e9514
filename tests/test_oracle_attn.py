"""The oracle's gated attention decode step (lio_attn_layer_decode) against an
independent numpy restatement of the same definition (CPU only). The
reference has no attention kernel and no vector for it, so this pins the
oracle's own arithmetic: RMSNorm per head, NeoX rotate-half RoPE, the fp16
cache round trip, softmax over positions 0..pos, the sigmoid output gate."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_close, rng


def _np_attn_step(w, x, kc, vc, pos, oracle_mod):
    from leaninfer_b200 import synth  # noqa: F401
    D, Hq, Hkv, rd = w["head_dim"], w["n_q_heads"], w["n_kv_heads"], w["rope_dim"]
    eps = w["eps"]
    n = x.shape[0]
    p = oracle_mod.rms_norm_matmul(w["wtype"], x, w["in_norm_w"], w["w_in"], 2 * Hq * D + 2 * Hkv * D, eps)
    p = p.astype(np.float64)

    def norm_rope(v, g, ps):
        v = v * g / np.sqrt(np.mean(v * v) + eps)
        half = rd // 2
        f = ps * w["rope_theta"] ** (-2.0 * np.arange(half) / rd)
        c, s = np.cos(f), np.sin(f)
        x1, x2 = v[:half].copy(), v[half:rd].copy()
        v[:half], v[half:rd] = x1 * c - x2 * s, x2 * c + x1 * s
        return v

    kc = kc.copy()
    vc = vc.copy()
    og = np.zeros((n, Hq * D))
    for s in range(n):
        ps = int(pos[s])
        for j in range(Hkv):
            k = norm_rope(p[s, 2 * Hq * D + j * D:2 * Hq * D + (j + 1) * D].copy(), w["k_norm_w"], ps)
            kc[s, ps, j] = k.astype(np.float32).astype(np.float16).view(np.uint16)
            vv = p[s, 2 * Hq * D + Hkv * D + j * D:2 * Hq * D + Hkv * D + (j + 1) * D]
            vc[s, ps, j] = vv.astype(np.float32).astype(np.float16).view(np.uint16)
        for h in range(Hq):
            j = h // (Hq // Hkv)
            q = norm_rope(p[s, h * D:(h + 1) * D].copy(), w["q_norm_w"], ps)
            K = kc[s, :ps + 1, j].view(np.float16).astype(np.float64)
            V = vc[s, :ps + 1, j].view(np.float16).astype(np.float64)
            sc = K @ q / np.sqrt(D)
            e = np.exp(sc - sc.max())
            o = (e / e.sum()) @ V
            gate = p[s, Hq * D + h * D:Hq * D + (h + 1) * D]
            og[s, h * D:(h + 1) * D] = o / (1 + np.exp(-gate))
    y = oracle_mod.rms_norm_matmul(w["wtype"], og.astype(np.float32), None, w["w_out"], w["hidden"])
    return y, kc, vc


@pytest.mark.parametrize("G", [1, 3])
def test_oracle_attn_step_matches_numpy(oracle_mod, G):
    from leaninfer_b200 import synth
    r = rng(55 + G)
    w = synth.attn_layer(r, hidden=256, n_q_heads=2 * G, n_kv_heads=2, rope_dim=32, wtype=8)
    L, keep = oracle_mod.make_attn_layer(w)
    inp = synth.attn_inputs(r, 3, w, 40, pos=np.array([0, 17, 39], np.int32))
    kc, vc = inp["k_cache"].copy(), inp["v_cache"].copy()
    y = oracle_mod.attn_layer_decode(L, keep, inp["x"], kc, vc, inp["pos"])
    y_np, kc_np, vc_np = _np_attn_step(w, inp["x"], inp["k_cache"], inp["v_cache"], inp["pos"], oracle_mod)
    assert_close(y, y_np, 1e-5, "y")
    # the cache rows: the same f16 values but for a rare double -> f32 -> f16 rounding tie
    assert np.mean(kc != kc_np) < 1e-3 and np.array_equal(vc, vc_np)


def test_fp32_to_fp16_matches_numpy(oracle_mod):
    r = rng(9)
    vals = np.concatenate([r.standard_normal(2000) * 10.0 ** r.integers(-8, 5, size=2000),
                           [0.0, -0.0, 65504.0, 65520.0, -65519.0, 6.1e-5, 5.96e-8, 2.9e-8, 1e-9]]).astype(np.float32)
    got = np.array([oracle_mod.fp32_to_fp16_bits(v) for v in vals], np.uint16)
    with np.errstate(over="ignore"):       # 65520 rounds to infinity, as it should
        want = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)
