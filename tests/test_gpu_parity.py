"""GPU parity of every C-ABI entry against the CPU oracle on identical seeded
inputs, and against the reference's own kernels (built from its sources into
oracle/_ref/) where they exist.

Tolerances: block decode bit-exact; fp32 outputs and fp32 state within a
normwise relative error of 1e-3 (max|got - ref| <= 1e-3 * max|ref|).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import GOLDEN, assert_close, max_rel_err, rng

pytestmark = pytest.mark.gpu
TOL = 1e-3
# Layer output y when the projections run on the tensor cores (f16 operands:
# X and the dequantized weights each rounded to f16 once, fp32 accumulation;
# about 4e-4 normwise per projection at hidden 4096, two projections composed
# through the recurrence). States and conv states keep TOL on every path.
TOL_Y_F16 = 2e-3


def T(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def N(t):
    return t.detach().cpu().numpy()


# --------------------------------------------------------------------------
# block decode
# --------------------------------------------------------------------------
@pytest.mark.parametrize("name,wtype,bs", [("q8_0", 8, 32), ("q4_k", 12, 256)])
def test_dequant_bit_exact_golden(cuda, name, wtype, bs):
    from leaninfer_b200 import ops
    f = np.load(GOLDEN / f"dequant_{name}.npz")
    n = f["blocks"].shape[0] * bs
    got = N(ops.dequantize(wtype, T(f["blocks"], cuda), n))
    assert np.array_equal(got.view(np.uint32), f["values"].view(np.uint32))


@pytest.mark.parametrize("wtype", [8, 12])
def test_dequant_bit_exact_random(cuda, oracle_mod, wtype):
    from leaninfer_b200 import ops, synth
    W = synth.random_weights(rng(3), wtype, 64, 4096)
    got = N(ops.dequantize(wtype, T(W, cuda), 64 * 4096))
    ref = oracle_mod.dequantize(wtype, W, 64 * 4096)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


# --------------------------------------------------------------------------
# reference dense entries (fp32 / fp16 weights)
# --------------------------------------------------------------------------
def _ref_gpu():
    from oracle import oracle
    if not oracle.REF_GPU.exists():
        return None
    lib = ctypes.CDLL(str(oracle.REF_GPU))
    return lib


@pytest.mark.parametrize("K,N_", [(896, 4864), (4096, 1000), (1000, 77)])
def test_dense_matmul_and_swiglu(cuda, oracle_mod, K, N_):
    import torch
    from leaninfer_b200 import ops
    r = rng(K + N_)
    x = r.standard_normal(K).astype(np.float32)
    gamma = r.uniform(0.5, 1.5, K).astype(np.float32)
    Wg = (r.standard_normal((N_, K)) * 0.02).astype(np.float32)
    Wu = (r.standard_normal((N_, K)) * 0.02).astype(np.float32)
    dx, dg, dWg, dWu = (T(a, cuda) for a in (x, gamma, Wg, Wu))
    mm = N(ops.rms_norm_matmul_f32(dx, dg, dWg, 1e-6))
    assert_close(mm, oracle_mod.rms_norm_matmul(0, x, gamma, Wg, N_, 1e-6)[0], TOL, "matmul f32")
    sw = N(ops.rms_norm_swiglu_f32(dx, dg, dWg, dWu, 1e-6))
    assert_close(sw, oracle_mod.rms_norm_swiglu(0, x, gamma, Wg, Wu, N_, 1e-6)[0], TOL, "swiglu f32")
    Wg16, Wu16 = Wg.astype(np.float16), Wu.astype(np.float16)
    sw16 = N(ops.rms_norm_swiglu_f16(dx, dg, T(Wg16, cuda), T(Wu16, cuda), 1e-6))
    ref16 = oracle_mod.rms_norm_swiglu(1, x, gamma, Wg16, Wu16, N_, 1e-6, round_xn_f16=True)[0]
    assert_close(sw16, ref16, TOL, "swiglu f16")
    qkv = ops.rms_norm_qkv_f32(dx, dg, [dWg, dWu, dWg], 1e-6)
    assert_close(N(qkv[1]), oracle_mod.rms_norm_matmul(0, x, gamma, Wu, N_, 1e-6)[0], TOL, "qkv f32")
    # the same with the pointer arrays in device memory: the same arithmetic, bit for bit
    qkv_d = ops.rms_norm_qkv_f32(dx, dg, [dWg, dWu, dWg], 1e-6, device_arrays=True)
    for a, b in zip(qkv, qkv_d):
        assert np.array_equal(N(a), N(b))
    ref = _ref_gpu()
    if ref is not None and K % 4 == 0:
        # the reference's own kernel on the same device buffers
        out = torch.empty(N_, device=cuda)
        ref.li_launch_fused_rms_norm_swiglu_f32(*(ctypes.c_void_p(t.data_ptr()) for t in (dx, dg, dWg, dWu, out)),
                                                ctypes.c_int(K), ctypes.c_int(N_), ctypes.c_float(1e-6),
                                                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        assert max_rel_err(sw, N(out)) <= TOL


def test_qkv_f32_pointer_arrays_on_different_sides_are_refused(cuda):
    import torch
    from leaninfer_b200 import _lib
    lib = _lib.load()
    x = torch.ones(256, device=cuda)
    W = torch.zeros(4, 256, device=cuda)
    out = torch.empty(4, device=cuda)
    host_w = (ctypes.c_void_p * 3)(*[W.data_ptr()] * 3)
    dev_d = torch.tensor([out.data_ptr()] * 3, dtype=torch.int64, device=cuda)
    lib.li_launch_fused_rms_norm_qkv_f32(x.data_ptr(), x.data_ptr(), host_w,
                                         ctypes.cast(ctypes.c_void_p(dev_d.data_ptr()),
                                                     ctypes.POINTER(ctypes.c_void_p)),
                                         256, 4, 1e-6, None)
    assert lib.li_get_last_error() == 2001


def test_silu_gate(cuda, oracle_mod):
    import torch
    from leaninfer_b200 import ops
    r = rng(77)
    o = r.standard_normal((64, 128)).astype(np.float32)
    z = r.standard_normal((64, 128)).astype(np.float32)
    gamma = r.uniform(0.5, 1.5, 128).astype(np.float32)
    got = N(ops.rms_norm_silu_gate_f32(T(o, cuda), T(z, cuda), T(gamma, cuda), 1e-6))
    assert_close(got, oracle_mod.silu_gate(o, z, gamma, 1e-6), TOL, "gate")
    ref = _ref_gpu()
    if ref is not None:
        out = torch.empty(64, 128, device=cuda)
        ref.li_launch_fused_rms_norm_silu_gate_f32(
            *(ctypes.c_void_p(t.data_ptr()) for t in (T(o, cuda), T(z, cuda), T(gamma, cuda), out)),
            ctypes.c_int(128), ctypes.c_int(64), ctypes.c_float(1e-6),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        assert max_rel_err(got, N(out)) <= 1e-5


# --------------------------------------------------------------------------
# quantized GEMVs
# --------------------------------------------------------------------------
@pytest.mark.parametrize("wtype", [8, 12])
def test_qkv_q_config1_shapes(cuda, oracle_mod, wtype):
    """RMSNorm + Q/K/V projections, K=2048 -> 2048/512/512 (the Q8_0 workload)."""
    from leaninfer_b200 import ops, synth
    r = rng(100 + wtype)
    K = 2048
    x = r.standard_normal((1, K)).astype(np.float32)
    gamma = r.uniform(0.5, 1.5, K).astype(np.float32)
    Ws = [synth.random_weights(r, wtype, n, K) for n in (2048, 512, 512)]
    got = ops.rms_norm_qkv_q(wtype, T(x, cuda), T(gamma, cuda), *(T(w, cuda) for w in Ws), 2048, 512, 512, 1e-6)
    for g, w, n, name in zip(got, Ws, (2048, 512, 512), "qkv"):
        assert_close(N(g), oracle_mod.rms_norm_matmul(wtype, x, gamma, w, n, 1e-6), TOL, f"{name} w{wtype}")


@pytest.mark.parametrize("wtype", [8, 12])
@pytest.mark.parametrize("n_rows", [1, 2, 3, 6, 8])
def test_matmul_q_shapes(cuda, oracle_mod, wtype, n_rows):
    """Up to 8 rows, K = 1024 (Q8_0) / 2048 (Q4_K) per unit per lane take the
    few-row kernel (K = 4096 here), the others the staged kernel."""
    from leaninfer_b200 import ops, synth
    r = rng(200 + wtype + n_rows)
    for K, N_ in [(256, 5), (4096, 1037), (12288, 512), (5120, 333)]:
        x = r.standard_normal((n_rows, K)).astype(np.float32)
        W = synth.random_weights(r, wtype, N_, K)
        got = N(ops.rms_norm_matmul_q(wtype, T(x, cuda), None, T(W, cuda), N_))
        assert_close(got, oracle_mod.rms_norm_matmul(wtype, x, None, W, N_), TOL, f"K={K} N={N_}")


@pytest.mark.parametrize("wtype", [8, 12])
@pytest.mark.parametrize("n_rows", [2, 5, 8, 32, 64, 256])
def test_ffn_q(cuda, oracle_mod, wtype, n_rows):
    """RMSNorm + SwiGLU gate/up + down, reduced width (K=1024, N=3072); from 3
    rows on the gate/up and down contractions run on the tensor cores (A tiles
    in tensor memory; at 256 rows the gate/up accumulators fill the TMEM and
    the A tiles go through shared memory)."""
    from leaninfer_b200 import ops, synth
    r = rng(300 + wtype + n_rows)
    K, N_ = 1024, 3072
    x = r.standard_normal((n_rows, K)).astype(np.float32)
    gamma = r.uniform(0.5, 1.5, K).astype(np.float32)
    Wg, Wu = synth.random_weights(r, wtype, N_, K), synth.random_weights(r, wtype, N_, K)
    Wd = synth.random_weights(r, wtype, K, N_)
    dx, dg = T(x, cuda), T(gamma, cuda)
    h = N(ops.rms_norm_swiglu_q(wtype, dx, dg, T(Wg, cuda), T(Wu, cuda), N_))
    assert_close(h, oracle_mod.rms_norm_swiglu(wtype, x, gamma, Wg, Wu, N_), TOL, "swiglu")
    y = N(ops.ffn_q(wtype, dx, dg, T(Wg, cuda), T(Wu, cuda), T(Wd, cuda), N_))
    assert_close(y, oracle_mod.ffn(wtype, x, gamma, Wg, Wu, Wd, N_), TOL, "ffn")


# --------------------------------------------------------------------------
# recurrence (reference layouts)
# --------------------------------------------------------------------------
@pytest.mark.parametrize("case", ["d128", "d64"])
def test_recurrence_golden(cuda, case):
    from leaninfer_b200 import ops
    f = np.load(GOLDEN / "gdr_recurrent.npz")
    g = {k[len(case) + 1:]: f[k] for k in f.files if k.startswith(case + "_")}
    B, T_, H, D = (int(v) for v in g["dims"])
    out, st = ops.deltanet_recurrent_f32(
        *(T(g[n], cuda) for n in ("q", "k", "v", "g", "beta_logit", "state")), head_dim=D, n_tokens=T_,
        n_heads=H, gqa_ratio=1, repeat_type=0, n_seqs=B, vnb1=D, vnb2=D * T_, vnb3=D * T_ * H)
    assert_close(N(out).reshape(B, T_, H, D), g["out"], TOL, "outputs")
    assert_close(N(st).reshape(B, H, D, D), g["state_out"], TOL, "state")


def _rec_inputs(r, B, T_, H, gqa, D):
    Hk = H // gqa
    q = r.standard_normal((B, Hk, T_, D)).astype(np.float32)
    k = r.standard_normal((B, Hk, T_, D)).astype(np.float32)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = r.standard_normal((B, H, T_, D)).astype(np.float32)
    g = (-np.log1p(np.exp(r.standard_normal((B, T_, H))))).astype(np.float32)
    beta = r.standard_normal((B, T_, H)).astype(np.float32)
    s0 = r.normal(0, 0.02, (B, H, D, D)).astype(np.float32)
    return q, k, v, g, beta, s0


@pytest.mark.parametrize("D,gqa,repeat_type", [(128, 2, 0), (128, 2, 1), (64, 1, 0), (128, 4, 1)])
def test_recurrence_gqa_and_tokens(cuda, oracle_mod, D, gqa, repeat_type):
    from leaninfer_b200 import ops
    r = rng(D + 10 * gqa + repeat_type)
    B, T_, H = 3, 6, 8
    q, k, v, g, beta, s0 = _rec_inputs(r, B, T_, H, gqa, D)
    kw = dict(n_tokens=T_, n_heads=H, repeat_type=repeat_type, n_seqs=B, vnb1=D, vnb2=D * T_, vnb3=D * T_ * H)
    out, st = ops.deltanet_recurrent_f32(*(T(a, cuda) for a in (q, k, v, g, beta, s0)), head_dim=D,
                                         gqa_ratio=gqa, **kw)
    ro, rs, _ = oracle_mod.deltanet_recurrent(q, k, v, g, beta, s0, D=D, gqa=gqa, **kw)
    assert_close(N(out), ro, TOL, "outputs")
    assert_close(N(st).reshape(-1), rs, TOL, "state")
    # in place: state_out == state_in
    ds = T(s0, cuda)
    ops.deltanet_recurrent_f32(*(T(a, cuda) for a in (q, k, v, g, beta)), ds, head_dim=D, gqa_ratio=gqa,
                               state_out=ds, **kw)
    assert_close(N(ds).reshape(-1), rs, TOL, "in-place state")


def test_recurrent_out_legacy_entry(cuda, oracle_mod):
    """li_launch_fused_deltanet_recurrent_out_f32: outputs + state in dst as
    the reference lays them out; proj_out = W_out . o (all D terms)."""
    from leaninfer_b200 import ops
    r = rng(4242)
    B, T_, H, gqa, D, hidden = 1, 3, 4, 2, 128, 320
    q, k, v, g, beta, s0 = _rec_inputs(r, B, T_, H, gqa, D)
    W = (r.standard_normal((hidden, H * D)) * 0.05).astype(np.float32)
    kw = dict(n_tokens=T_, n_heads=H, repeat_type=0, n_seqs=B, vnb1=D, vnb2=D * T_, vnb3=D * T_ * H)
    dst, proj = ops.deltanet_recurrent_out_f32(*(T(a, cuda) for a in (q, k, v, g, beta, s0, W)), head_dim=D,
                                               gqa_ratio=gqa, hidden_dim=hidden, **kw)
    ro, rs, rp = oracle_mod.deltanet_recurrent(q, k, v, g, beta, s0, D=D, gqa=gqa, W_out=W, hidden=hidden, **kw)
    dst = N(dst)
    assert_close(dst[:ro.size], ro, TOL, "outputs")
    assert_close(dst[ro.size:], rs, TOL, "state")
    assert_close(N(proj), rp, TOL, "proj_out")



def test_recurrent_vs_reference_kernel_one_token(cuda, oracle_mod):
    """Per-head outputs and state against the reference's own kernel, built
    from its sources (oracle/_ref). One token only: for n_tokens > 1 the
    reference kernel overwrites its shared q/k (cuda/leaninfer-fused-deltanet.cu
    :219-222) with no barrier after the previous token's state update reads
    them (:281-288), so its multi-token results depend on warp timing. Its
    proj_out is not compared: it sums D/32 of the terms per head (:264-279)."""
    import torch
    from leaninfer_b200 import ops
    ref = _ref_gpu()
    if ref is None:
        pytest.skip("reference kernels not built (oracle/_ref)")
    r = rng(4343)
    B, T_, H, gqa, D, hidden = 2, 1, 8, 2, 128, 256
    q, k, v, g, beta, s0 = _rec_inputs(r, B, T_, H, gqa, D)
    W = (r.standard_normal((hidden, H * D)) * 0.05).astype(np.float32)
    kw = dict(n_tokens=T_, n_heads=H, repeat_type=0, n_seqs=B, vnb1=D, vnb2=D * T_, vnb3=D * T_ * H)
    dst, _ = ops.deltanet_recurrent_out_f32(*(T(a, cuda) for a in (q, k, v, g, beta, s0, W)), head_dim=D,
                                            gqa_ratio=gqa, hidden_dim=hidden, **kw)
    dst = N(dst)
    n_out = B * T_ * H * D
    dq, dk, dv, dgg, db, ds, dW = (T(a, cuda) for a in (q, k, v, g, beta, s0, W))
    rdst = torch.empty(n_out + s0.size, device=cuda)
    rproj = torch.empty(hidden * T_, device=cuda)
    fn = ref.li_launch_fused_deltanet_recurrent_out_f32
    fn.argtypes = [ctypes.c_void_p] * 9 + [ctypes.c_int64] * 4 + [ctypes.c_int, ctypes.c_int64, ctypes.c_int64,
                                                                 ctypes.c_size_t, ctypes.c_size_t,
                                                                 ctypes.c_size_t, ctypes.c_void_p]
    fn(*(t.data_ptr() for t in (dq, dk, dv, dgg, db, ds, dW, rdst, rproj)), D, T_, H, gqa, 0, B, hidden,
       D, D * T_, D * T_ * H, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    rd = N(rdst)
    assert_close(dst[:n_out], rd[:n_out], 1e-4, "vs reference kernel outputs")
    assert_close(dst[n_out:], rd[n_out:], 1e-4, "vs reference kernel state")


# --------------------------------------------------------------------------
# fused DeltaNet decode layer
# --------------------------------------------------------------------------
def _layer(cuda, w, repeat_type=0, in_norm_w=None):
    from leaninfer_b200 import ops
    return ops.DeltaNetLayerDecode(
        hidden=w["hidden"], n_k_heads=w["n_k_heads"], n_v_heads=w["n_v_heads"], head_dim=w["head_dim"],
        w_in=T(w["w_in"], cuda), conv_w=T(w["conv_w"], cuda), a_log=T(w["a_log"], cuda),
        dt_bias=T(w["dt_bias"], cuda), norm_w=T(w["norm_w"], cuda), w_out=T(w["w_out"], cuda),
        w_in_type=w["wtype"], w_out_type=w["wtype"], repeat_type=repeat_type,
        in_norm_w=None if in_norm_w is None else T(in_norm_w, cuda))


@pytest.mark.parametrize("wtype,B,hidden,Hk,Hv,repeat_type", [
    (12, 2, 1024, 4, 8, 0),
    (8, 3, 1024, 2, 8, 1),
    (12, 1, 4096, 16, 32, 0),      # the decode workload's layer shape
    (12, 3, 4096, 16, 32, 1),      # few-row SIMT projections at the layer shape
    (12, 8, 4096, 16, 32, 0),
    (12, 5, 1024, 4, 8, 0),        # tensor-core projections from 3 sequences on
    (12, 8, 1024, 4, 8, 0),
    (8, 16, 1024, 2, 8, 1),
    (12, 64, 4096, 16, 32, 0),     # the decode workload: layer shape and batch
    (8, 40, 1024, 4, 16, 1),       # 640 (sequence, head) items, k-heads repeated by tiling
])
def test_layer_decode_steps(cuda, oracle_mod, wtype, B, hidden, Hk, Hv, repeat_type):
    import torch
    from leaninfer_b200 import synth
    r = rng(500 + B + hidden)
    w = synth.deltanet_layer(r, hidden=hidden, n_k_heads=Hk, n_v_heads=Hv, wtype=wtype)
    layer = _layer(cuda, w, repeat_type)
    L, keep = oracle_mod.make_layer(w, repeat_type=repeat_type)
    inp = synth.deltanet_inputs(r, B, w)
    cs_ref, st_ref = inp["conv_state"].copy(), inp["state"].copy()
    cs, st = T(inp["conv_state"], cuda), T(inp["state"], cuda)
    for step in range(3):
        x = (r.standard_normal((B, hidden)) * synth.DELTANET_X_SCALE).astype(np.float32)
        y = torch.empty(B, hidden, device=cuda)
        layer.step(T(x, cuda), y, cs, st)
        y_ref = oracle_mod.deltanet_layer_decode(L, keep, x, cs_ref, st_ref)
        assert_close(N(y), y_ref, TOL_Y_F16 if B >= 3 else TOL, f"y step {step}")
        assert_close(N(cs), cs_ref, TOL, f"conv state step {step}")
        assert_close(N(st), st_ref, TOL, f"state step {step}")


@pytest.mark.parametrize("wtype,B,hidden,Hk,Hv", [
    (12, 2, 1024, 4, 8),           # SIMT projections
    (8, 5, 1024, 2, 8),            # tensor-core projections
    (12, 64, 4096, 16, 32),        # the decode workload
])
def test_layer_decode_f16_state(cuda, oracle_mod, wtype, B, hidden, Hk, Hv):
    """fp16 state storage: the oracle's step with its state rounded to fp16
    after every step (saturated at +-65504). States that round differently
    differ by one fp16 step (2^-10 relative); 2e-3 normwise allows that."""
    import torch
    from leaninfer_b200 import synth
    r = rng(700 + B + hidden)
    w = synth.deltanet_layer(r, hidden=hidden, n_k_heads=Hk, n_v_heads=Hv, wtype=wtype)
    layer = _layer(cuda, w, 0)
    L, keep = oracle_mod.make_layer(w, repeat_type=0)
    inp = synth.deltanet_inputs(r, B, w)
    f16 = lambda a: np.clip(a, -65504, 65504).astype(np.float16).astype(np.float32)
    cs_ref, st_ref = inp["conv_state"].copy(), f16(inp["state"])
    cs, st = T(inp["conv_state"], cuda), T(st_ref, cuda).half()
    for step in range(3):
        x = (r.standard_normal((B, hidden)) * synth.DELTANET_X_SCALE).astype(np.float32)
        y = torch.empty(B, hidden, device=cuda)
        layer.step(T(x, cuda), y, cs, st)
        y_ref = oracle_mod.deltanet_layer_decode(L, keep, x, cs_ref, st_ref)
        st_ref[...] = f16(st_ref)
        assert_close(N(y), y_ref, 2e-3, f"y step {step}")
        assert_close(N(cs), cs_ref, TOL, f"conv state step {step}")
        assert_close(N(st.float()), st_ref, 2e-3, f"state step {step}")


def test_layer_decode_with_input_norm(cuda, oracle_mod):
    import torch
    from leaninfer_b200 import synth
    r = rng(77)
    w = synth.deltanet_layer(r, hidden=1024, n_k_heads=4, n_v_heads=8)
    g = r.uniform(0.5, 1.5, 1024).astype(np.float32)
    layer = _layer(cuda, w, in_norm_w=g)
    L, keep = oracle_mod.make_layer(w, in_norm_w=g)
    inp = synth.deltanet_inputs(r, 2, w)
    x = r.standard_normal((2, 1024)).astype(np.float32)
    cs, st = T(inp["conv_state"], cuda), T(inp["state"], cuda)
    y = torch.empty(2, 1024, device=cuda)
    layer.step(T(x, cuda), y, cs, st)
    y_ref = oracle_mod.deltanet_layer_decode(L, keep, x, inp["conv_state"], inp["state"])
    assert_close(N(y), y_ref, TOL, "y")


def test_device_status_clean(cuda):
    from leaninfer_b200 import ops
    assert ops.device_status() == 0


# --------------------------------------------------------------------------
# chunked (WY) prefill on the tensor cores
# --------------------------------------------------------------------------
def _prefill_inputs(r, n_tok, Hk, Hv, D=128):
    """Config-4 value distributions: q, k L2-normalised, v N(0,1) (bf16);
    beta = sigmoid(N(0,1)); a = exp(-softplus(N(0,1)) * exp(N(0,0.5))), g = log a;
    state N(0, 0.02)."""
    def bf16_bits(x):
        u = np.ascontiguousarray(x, np.float32).view(np.uint32)
        return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)   # round to nearest even
    q = r.standard_normal((n_tok, Hk, D)).astype(np.float32)
    k = r.standard_normal((n_tok, Hk, D)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = r.standard_normal((n_tok, Hv, D)).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-r.standard_normal((n_tok, Hv))))).astype(np.float32)
    g = (-np.log1p(np.exp(r.standard_normal((n_tok, Hv)))) * np.exp(r.normal(0.0, 0.5, (n_tok, Hv)))).astype(np.float32)
    state = r.normal(0.0, 0.02, (Hv, D, D)).astype(np.float32)
    return bf16_bits(q), bf16_bits(k), bf16_bits(v), g, beta, state


@pytest.mark.parametrize("n_tok,Hk,Hv", [(64, 1, 1), (130, 2, 4), (1000, 2, 2), (2048, 1, 2)])
def test_chunk_prefill_vs_token_recurrence(cuda, oracle_mod, n_tok, Hk, Hv):
    """The tensor-core chunked prefill against the oracle's token-by-token
    recurrence (double precision) on the same bf16 inputs: outputs and final
    state within 2e-2 normwise (bf16 operands, fp32 accumulation); ragged T
    covers the zero-padded last chunk."""
    import torch
    from leaninfer_b200 import ops
    r = rng(900 + n_tok + Hv)
    q, k, v, g, beta, state = _prefill_inputs(r, n_tok, Hk, Hv)
    scale = 128 ** -0.5
    st_ref = state.copy()
    o_ref = oracle_mod.gdr_prefill(q, k, v, g, beta, st_ref, scale)
    tb = lambda a: torch.from_numpy(a.view(np.int16)).to(cuda).view(torch.bfloat16)
    st = T(state, cuda)
    o = ops.deltanet_chunk_prefill_bf16(tb(q), tb(k), tb(v), T(g, cuda), T(beta, cuda), st, scale)
    torch.cuda.synchronize()
    assert_close(N(o), o_ref, 2e-2, "prefill outputs")
    assert_close(N(st), st_ref, 2e-2, "prefill final state")


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 1024), (512, 256, 4096)])
def test_gemm_bf16_vs_torch_fp32(cuda, M, N, K):
    """The tensor-core bf16 GEMM (out-projection of the prefill) against a
    torch fp32 matmul of the same bf16 values: the products are exact and the
    sums fp32, so only the summation order differs (1e-4 normwise)."""
    import torch
    from leaninfer_b200 import ops
    g = torch.Generator(device=cuda)
    g.manual_seed(M + N + K)
    A = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    W = (0.02 * torch.randn(N, K, device=cuda, generator=g)).bfloat16()
    C = ops.gemm_bf16(A, W)
    ref = A.float() @ W.float().T
    torch.cuda.synchronize()
    assert_close(N_(C), N_(ref), 1e-4, "bf16 gemm")


def test_gated_rmsnorm_bf16_vs_oracle(cuda, oracle_mod):
    from leaninfer_b200 import ops
    r = rng(4242)
    o = r.standard_normal((300, 128)).astype(np.float32)
    z = r.standard_normal((300, 128)).astype(np.float32)
    gamma = r.uniform(0.5, 1.5, 128).astype(np.float32)
    got = ops.gated_rmsnorm_bf16(T(o, cuda), T(z, cuda), T(gamma, cuda)).float()
    assert_close(N_(got), oracle_mod.silu_gate(o, z, gamma), 8e-3, "gated rmsnorm (bf16 output)")


def N_(t):
    return t.detach().float().cpu().numpy()
