"""The CPU oracle pinned against the committed golden fixtures (CPU only).

Fixtures (tests/golden/make_golden.py): gguf-py 0.19.0 block decode,
flash-linear-attention's naive recurrent and chunked gated delta rule, and
the reference's own cpu_rms_norm_swiglu (cuda/benchmark_fused.cu:99-121).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN, assert_close


@pytest.mark.parametrize("name,wtype,bs", [("q8_0", 8, 32), ("q4_k", 12, 256)])
def test_dequant_bit_exact_vs_gguf(oracle_mod, name, wtype, bs):
    f = np.load(GOLDEN / f"dequant_{name}.npz")
    blocks, values = f["blocks"], f["values"]
    got = oracle_mod.dequantize(wtype, blocks, blocks.shape[0] * bs)
    assert got.view(np.uint32).tolist() == values.view(np.uint32).tolist() or \
        np.array_equal(got.view(np.uint32), values.view(np.uint32))


@pytest.mark.parametrize("case", ["d128", "d64"])
def test_recurrence_vs_fla_naive(oracle_mod, case):
    f = np.load(GOLDEN / "gdr_recurrent.npz")
    g = {k[len(case) + 1:]: f[k] for k in f.files if k.startswith(case + "_")}
    B, T, H, D = (int(v) for v in g["dims"])
    out, st, _ = oracle_mod.deltanet_recurrent(
        g["q"], g["k"], g["v"], g["g"], g["beta_logit"], g["state"], D=D, n_tokens=T, n_heads=H, gqa=1,
        repeat_type=0, n_seqs=B, vnb1=D, vnb2=D * T, vnb3=D * T * H)
    assert_close(out.reshape(B, T, H, D), g["out"], 1e-5, "outputs")
    assert_close(st.reshape(B, H, D, D), g["state_out"], 1e-5, "state")


def test_sequential_prefill_matches_fla_chunk_form(oracle_mod):
    f = np.load(GOLDEN / "gdr_chunk.npz")
    T, H, D = f["out"].shape
    state = f["state"].astype(np.float32).copy()
    o = oracle_mod.gdr_prefill(f["q"], f["k"], f["v"], f["g"], f["beta"], state, D ** -0.5)
    assert_close(o, f["out"], 1e-5, "chunk-form outputs")
    assert_close(state, f["state_out"], 1e-5, "chunk-form final state")


def test_f32_swiglu_vs_reference_cpu_function(oracle_mod):
    f = np.load(GOLDEN / "ref_cpu_swiglu.npz")
    got = oracle_mod.rms_norm_swiglu(0, f["x"], f["gamma"], f["Wg"], f["Wu"], f["Wg"].shape[0], float(f["eps"]))
    # the reference accumulates in fp32 (and uses 1/sqrtf): ~1e-6 from the exact value
    assert_close(got[0], f["out"], 1e-5, "swiglu")


def test_gate_matches_patch_cpu_fallback(oracle_mod):
    """Gated RMSNorm vs a direct restatement of the ggml CPU fallback of
    scripts/patch_fused_gate.sh:89-110 in fp32."""
    from conftest import rng
    r = rng(5)
    o = r.standard_normal((6, 128)).astype(np.float32)
    z = r.standard_normal((6, 128)).astype(np.float32)
    gamma = r.uniform(0.5, 1.5, 128).astype(np.float32)
    ref = np.empty_like(o)
    for i in range(6):
        rms = np.float32(1.0) / np.sqrt(np.float32((o[i] * o[i]).sum(dtype=np.float32) / 128) + np.float32(1e-6))
        ref[i] = (z[i] / (1 + np.exp(-z[i]))) * (o[i] * gamma * rms)
    assert_close(oracle_mod.silu_gate(o, z, gamma, 1e-6), ref, 1e-5, "gate")


def test_q4k_matmul_is_dequant_then_dot(oracle_mod):
    from conftest import rng
    from leaninfer_b200 import synth
    r = rng(9)
    W = synth.random_q4_k(r, 8, 512)
    x = r.standard_normal((2, 512)).astype(np.float32)
    deq = oracle_mod.dequantize(12, W, 8 * 512).reshape(8, 512).astype(np.float64)
    ref = x.astype(np.float64) @ deq.T
    assert_close(oracle_mod.rms_norm_matmul(12, x, None, W, 8), ref, 1e-6, "q4k matmul")
