"""GPU parity at the full sizes the benchmark times, through the C ABI.

The parity file covers every entry at reduced widths; these cases run the
exact shapes of the benchmarked workloads against the oracle:

- the SwiGLU FFN 4096 -> 12288 -> 4096 (Q4_K and Q8_0) at 1 row (few-row
  SwiGLU GEMV + staged down GEMV with K = 12288), 32 rows (X-stationary
  tensor-core GEMMs) and 64 rows (one-tile tensor-core GEMMs);
- the chunked prefill of one 8192-token sequence with 16 k-heads and 32
  v-heads, composed with the bf16 gated RMSNorm and the bf16 4096 x 4096
  out-projection;
- the bf16 GEMM alone at 8192 x 4096 x 4096.

Besides the normwise error held to the tolerance, each case reports the
elementwise relative error over the elements above 1e-3 of the largest
magnitude (printed; run with -s to see it).
"""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import assert_close, elementwise_rel_err, max_rel_err, rng

pytestmark = pytest.mark.gpu
TOL = 1e-3


def T(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def N(t):
    return t.detach().float().cpu().numpy()


def report(case: str, got, ref) -> tuple[float, float]:
    nw, ew = max_rel_err(got, ref), elementwise_rel_err(got, ref)
    print(json.dumps({"case": case, "normwise": nw, "elementwise_above_1e-3_max": ew}))
    return nw, ew


@pytest.mark.parametrize("wtype", [12, 8])
@pytest.mark.parametrize("n_rows", [1, 32, 64])
def test_ffn_full_width(cuda, oracle_mod, wtype, n_rows):
    """RMSNorm + SwiGLU gate/up 4096 -> 12288 and down 12288 -> 4096 at the
    FFN workload's shape; x ~ N(0,1), gamma ~ U(0.5,1.5), random codes."""
    from leaninfer_b200 import ops, synth
    r = rng(7000 + 100 * wtype + n_rows)
    K, N_ = 4096, 12288
    x = r.standard_normal((n_rows, K)).astype(np.float32)
    gamma = r.uniform(0.5, 1.5, K).astype(np.float32)
    Wg, Wu = synth.random_weights(r, wtype, N_, K), synth.random_weights(r, wtype, N_, K)
    Wd = synth.random_weights(r, wtype, K, N_)
    dx, dg, dWg, dWu, dWd = T(x, cuda), T(gamma, cuda), T(Wg, cuda), T(Wu, cuda), T(Wd, cuda)
    h = N(ops.rms_norm_swiglu_q(wtype, dx, dg, dWg, dWu, N_))
    h_ref = oracle_mod.rms_norm_swiglu(wtype, x, gamma, Wg, Wu, N_)
    report(f"swiglu w{wtype} rows{n_rows}", h, h_ref)
    assert_close(h, h_ref, TOL, "swiglu")
    y = N(ops.ffn_q(wtype, dx, dg, dWg, dWu, dWd, N_))
    y_ref = oracle_mod.ffn(wtype, x, gamma, Wg, Wu, Wd, N_)
    report(f"ffn w{wtype} rows{n_rows}", y, y_ref)
    assert_close(y, y_ref, TOL, "ffn")


def test_gemm_bf16_full_size(cuda):
    """The prefill out-projection GEMM at its benchmarked size (8192 tokens x
    4096 x 4096) against a torch fp32 matmul of the same bf16 values."""
    import torch
    from leaninfer_b200 import ops
    g = torch.Generator(device=cuda)
    g.manual_seed(8192)
    A = torch.randn(8192, 4096, device=cuda, generator=g).bfloat16()
    W = (0.02 * torch.randn(4096, 4096, device=cuda, generator=g)).bfloat16()
    C = ops.gemm_bf16(A, W)
    ref = A.float() @ W.float().T
    torch.cuda.synchronize()
    got, want = N(C), N(ref)
    report("gemm_bf16 8192x4096x4096", got, want)
    assert_close(got, want, 1e-4, "bf16 gemm")


def test_prefill_chain_full_size(cuda, oracle_mod):
    """One 8192-token sequence, 16 k-heads, 32 v-heads, head_dim 128: chunked
    prefill -> bf16 gated RMSNorm -> bf16 out-projection 4096 -> 4096, against
    the oracle's token-by-token recurrence (double precision), its gated
    RMSNorm and an fp32 matmul with the same bf16 weights. Outputs and final
    state within 2e-2 normwise (bf16 operands)."""
    import torch
    from leaninfer_b200 import ops
    from test_gpu_parity import _prefill_inputs
    r = rng(8192)
    Tn, Hk, Hv, D = 8192, 16, 32, 128
    q, k, v, g, beta, state = _prefill_inputs(r, Tn, Hk, Hv, D)
    z = r.standard_normal((Tn, Hv * D)).astype(np.float32)
    gamma = r.uniform(0.5, 1.5, D).astype(np.float32)
    scale = D ** -0.5
    st_ref = state.copy()
    o_ref = oracle_mod.gdr_prefill(q, k, v, g, beta, st_ref, scale)            # [T, Hv, D]
    tb = lambda a: torch.from_numpy(a.view(np.int16)).to(cuda).view(torch.bfloat16)
    gw = torch.Generator(device=cuda)
    gw.manual_seed(4096)
    w_out = (0.02 * torch.randn(4096, Hv * D, device=cuda, generator=gw)).bfloat16()
    st = T(state, cuda)
    o = ops.deltanet_chunk_prefill_bf16(tb(q), tb(k), tb(v), T(g, cuda), T(beta, cuda), st, scale)
    og = ops.gated_rmsnorm_bf16(o.view(Tn * Hv, D), T(z, cuda).view(Tn * Hv, D), T(gamma, cuda))
    y = ops.gemm_bf16(og.view(Tn, Hv * D), w_out)
    torch.cuda.synchronize()
    report("prefill o T8192", N(o), o_ref)
    assert_close(N(o), o_ref, 2e-2, "prefill outputs")
    report("prefill state T8192", N(st), st_ref)
    assert_close(N(st), st_ref, 2e-2, "prefill final state")
    og_ref = oracle_mod.silu_gate(o_ref.reshape(Tn * Hv, D), z.reshape(Tn * Hv, D), gamma)
    y_ref = (torch.from_numpy(og_ref.reshape(Tn, Hv * D)).to(cuda) @ w_out.float().T)
    torch.cuda.synchronize()
    report("prefill chain y T8192", N(y), N(y_ref))
    assert_close(N(y), N(y_ref), 2e-2, "prefill chain out-projection")


def test_bounded_wait_gives_up_and_reports(cuda):
    """A wait that can never complete gives up after its limit, the kernel
    returns by itself, li_device_status() reports LI_ERR_TIMEOUT once (the
    read clears it), and the GPU context stays usable: a block decode right
    after is still bit-exact."""
    import ctypes

    import torch
    from leaninfer_b200 import _lib, ops, synth
    lib = _lib.load()
    assert lib.li_device_status() == 0
    elapsed = torch.zeros(1, dtype=torch.int64, device=cuda)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.li_selftest_bounded_wait(2000, ctypes.c_void_p(elapsed.data_ptr()), stream) == 0
    assert lib.li_device_status() == 2006                  # LI_ERR_TIMEOUT
    ns = int(elapsed.item())
    assert 2_000_000 <= ns < 1_000_000_000, ns             # it waited its 2 ms, and not much more
    assert lib.li_device_status() == 0                     # the read cleared the flag
    W = synth.random_weights(rng(5), 8, 16, 256)
    got = N(ops.dequantize(8, T(W, cuda), 16 * 256))
    from oracle import oracle
    assert np.array_equal(got.view(np.uint32), oracle.dequantize(8, W, 16 * 256).view(np.uint32))
