"""The ggml-style node dispatch (include/leaninfer-ggml.h): descriptor layout,
exported symbols and the checks that reject a node before any launch (CPU),
and on the GPU that each node runs exactly the entry it maps to."""
from __future__ import annotations

import ctypes
import subprocess

import numpy as np
import pytest

from conftest import ROOT, assert_close, rng



@pytest.fixture(scope="module")
def lib():
    from leaninfer_b200 import _lib, build
    build.build()
    return _lib.load()


def test_descriptor_layout_matches_c(tmp_path):
    """The ctypes mirror has the C struct's size and field offsets."""
    from leaninfer_b200._lib import GgmlTensor
    src = tmp_path / "t.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "leaninfer-ggml.h"\n'
                   'int main(void){printf("%zu %zu %zu %zu %zu %zu %zu\\n", sizeof(li_ggml_tensor),'
                   'offsetof(li_ggml_tensor, ne), offsetof(li_ggml_tensor, nb), offsetof(li_ggml_tensor, op),'
                   'offsetof(li_ggml_tensor, op_params), offsetof(li_ggml_tensor, src),'
                   'offsetof(li_ggml_tensor, data)); return 0;}\n')
    exe = tmp_path / "t"
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", f"-I{ROOT / 'include'}", str(src), "-o", str(exe)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    want = [ctypes.sizeof(GgmlTensor)] + [getattr(GgmlTensor, f).offset
                                          for f in ("ne", "nb", "op", "op_params", "src", "data")]
    assert got == want


def test_library_exports_the_dispatch(lib):
    assert hasattr(lib, "li_ggml_compute_forward") and hasattr(lib, "li_ggml_workspace_size")


def _fake_f32(shape, ptr=256):
    """A contiguous f32 descriptor over a pointer nothing dereferences."""
    from leaninfer_b200._lib import GgmlTensor
    d = GgmlTensor()
    d.type = 0
    dims = list(shape) + [1] * (4 - len(shape))
    s = 4
    for i in range(4):
        d.ne[i] = dims[i]
        d.nb[i] = s
        s *= dims[i]
    d.data = ptr
    return d


def _fake_quant(wtype, k, n, ptr=256):
    from leaninfer_b200._lib import GgmlTensor
    blk, size = (32, 34) if wtype == 8 else (256, 144)
    d = GgmlTensor()
    d.type = wtype
    rb = k // blk * size
    for i, (ne, nb) in enumerate([(k, size), (n, rb), (1, rb * n), (1, rb * n)]):
        d.ne[i] = ne
        d.nb[i] = nb
    d.data = ptr
    return d


def _run(lib, nd):
    return lib.li_ggml_compute_forward(ctypes.byref(nd), None, 0, None)


def test_rejects_before_launch(lib):
    """Every rejection happens on the host: these run without a GPU."""
    from leaninfer_b200 import ggml
    assert lib.li_ggml_compute_forward(None, None, 0, None) == 2001
    assert _run(lib, ggml.node(0, _fake_f32([8, 1]), [])) == 2003                    # no such op
    W, x = _fake_quant(12, 4096, 64), _fake_f32([4096, 2])
    assert _run(lib, ggml.node(ggml.OP_MUL_MAT, _fake_f32([64, 2]), [W, None])) == 2001
    f16 = _fake_f32([4096, 64])
    f16.type = 1
    assert _run(lib, ggml.node(ggml.OP_MUL_MAT, _fake_f32([64, 2]), [f16, x])) == 2003
    Wbad = _fake_quant(12, 4096, 64)
    Wbad.nb[1] += 16                                                                   # padded rows
    assert _run(lib, ggml.node(ggml.OP_MUL_MAT, _fake_f32([64, 2]), [Wbad, x])) == 2002
    assert _run(lib, ggml.node(ggml.OP_MUL_MAT, _fake_f32([64, 2]), [W, _fake_f32([2048, 2])])) == 2002
    assert _run(lib, ggml.node(ggml.OP_MUL_MAT, _fake_f32([64, 3]), [W, x])) == 2002  # rows differ
    xs = _fake_f32([4096, 2])
    xs.nb[1] *= 2                                                                      # strided rows
    assert _run(lib, ggml.node(ggml.OP_MUL_MAT, _fake_f32([64, 2]), [W, xs])) == 2002
    Wg8 = _fake_quant(8, 4096, 64)
    assert _run(lib, ggml.node(ggml.OP_FUSED_UP_GATE, _fake_f32([64, 2]), [W, Wg8, x])) == 2003
    o, z = _fake_f32([128, 8]), _fake_f32([128, 4])
    assert _run(lib, ggml.node(ggml.OP_FUSED_RMS_SILU_GATE, _fake_f32([128, 8]),
                               [o, z, _fake_f32([128])], [1e-6])) == 2002
    assert _run(lib, ggml.node(ggml.OP_FUSED_RMS_SILU_GATE, _fake_f32([128, 8]),
                               [o, _fake_f32([128, 8]), _fake_f32([64])], [1e-6])) == 2002


def _layer_node(hidden, Hk, Hv, D, B, wtype=12):
    from leaninfer_b200 import ggml
    C = 2 * Hk * D + Hv * D
    NI = C + Hv * D + 2 * Hv
    srcs = [_fake_f32([hidden, B]), _fake_f32([3, C, B]), _fake_f32([D, D, Hv, B]),
            _fake_quant(wtype, hidden, NI), _fake_f32([4, C]), _fake_f32([Hv]), _fake_f32([Hv]),
            _fake_f32([D]), _fake_quant(wtype, Hv * D, hidden), None]
    return ggml.node(ggml.OP_DELTANET_DECODE, _fake_f32([hidden, B]), srcs, [Hk, 0, 1e-6, 1e-6, 1e-6])


def test_layer_node_workspace_and_checks(lib):
    from leaninfer_b200._lib import DeltaNetLayer
    for B in (1, 3, 8, 64):
        nd = _layer_node(4096, 16, 32, 128, B)
        L = DeltaNetLayer(hidden=4096, n_k_heads=16, n_v_heads=32, head_dim=128, conv_kernel=4,
                          w_in_type=12, w_out_type=12)
        assert lib.li_ggml_workspace_size(ctypes.byref(nd)) == lib.li_deltanet_layer_workspace_size(
            ctypes.byref(L), B) > 0
    nd = _layer_node(4096, 16, 32, 128, 2)
    nd.src[3].contents.ne[1] -= 1                                                    # wrong W_in rows
    assert _run(lib, nd) == 2002 and lib.li_ggml_workspace_size(ctypes.byref(nd)) == 0
    nd = _layer_node(1024, 4, 8, 128, 2)
    nd.src[7] = ctypes.POINTER(type(nd))()                                            # no gamma
    assert _run(lib, nd) == 2001
    # an f16 state is accepted with f16 strides (and refused with f32 strides)
    nd = _layer_node(1024, 4, 8, 128, 2)
    st = nd.src[2].contents
    st.type = 1
    assert _run(lib, nd) == 2002
    for i, s in enumerate((2, 2 * 128, 2 * 128 * 128, 2 * 128 * 128 * 8)):
        st.nb[i] = s
    assert lib.li_ggml_workspace_size(ctypes.byref(nd)) > 0
    st.type = 30                                                                       # bf16: not a state type
    assert _run(lib, nd) == 2003


def test_nodes_reach_their_entry(lib):
    """A node that passes every check goes on to its entry's own checks: with
    the descriptors' addresses misaligned on purpose, the entry answers
    LI_ERR_MISALIGNED before any launch (so this runs without a GPU)."""
    from leaninfer_b200 import ggml
    W, x = _fake_quant(12, 4096, 64, ptr=258), _fake_f32([4096, 2], ptr=258)
    assert _run(lib, ggml.node(ggml.OP_MUL_MAT, _fake_f32([64, 2], ptr=258), [W, x])) == 2005
    for st_type in (0, 1):
        nd = _layer_node(1024, 4, 8, 128, 2)
        st = nd.src[2].contents
        if st_type == 1:
            st.type = 1
            for i, s in enumerate((2, 2 * 128, 2 * 128 * 128, 2 * 128 * 128 * 8)):
                st.nb[i] = s
        st.data = 258                                                                  # state misaligned
        ws = lib.li_ggml_workspace_size(ctypes.byref(nd))
        assert lib.li_ggml_compute_forward(ctypes.byref(nd), ctypes.c_void_p(256), ws, None) == 2005


# --------------------------------------------------------------------------
# GPU: a node gives exactly what its entry gives
# --------------------------------------------------------------------------
def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


@pytest.mark.gpu
@pytest.mark.parametrize("wtype", [8, 12])
def test_mul_mat_and_up_gate_nodes(cuda, oracle_mod, wtype):
    import torch
    from leaninfer_b200 import ggml, ops, synth
    r = rng(900 + wtype)
    K, N, M = 4096, 1037, 3
    x = r.standard_normal((M, K)).astype(np.float32)
    W, Wu = synth.random_weights(r, wtype, N, K), synth.random_weights(r, wtype, N, K)
    dx, dW, dWu = _t(x, cuda), _t(W, cuda), _t(Wu, cuda)
    y = torch.empty(M, N, device=cuda)
    nd = ggml.node(ggml.OP_MUL_MAT, ggml.f32_desc(y), [ggml.quant_desc(dW, wtype, K, N), ggml.f32_desc(dx)])
    assert ggml.compute_forward(nd) == 0
    ref = ops.rms_norm_matmul_q(wtype, dx, None, dW, N)
    torch.cuda.synchronize()
    assert torch.equal(y, ref)
    assert_close(y.cpu().numpy(), oracle_mod.rms_norm_matmul(wtype, x, None, W, N), 1e-3, "mul_mat node")
    h = torch.empty(M, N, device=cuda)
    nd = ggml.node(ggml.OP_FUSED_UP_GATE, ggml.f32_desc(h),
                   [ggml.quant_desc(dWu, wtype, K, N), ggml.quant_desc(dW, wtype, K, N), ggml.f32_desc(dx)])
    assert ggml.compute_forward(nd) == 0
    ref = ops.rms_norm_swiglu_q(wtype, dx, None, dW, dWu, N)   # gate = W, up = Wu
    torch.cuda.synchronize()
    assert torch.equal(h, ref)


@pytest.mark.gpu
def test_gate_node(cuda):
    import torch
    from leaninfer_b200 import ggml, ops
    r = rng(910)
    o, z = _t(r.standard_normal((64, 128)).astype(np.float32), cuda), _t(r.standard_normal((64, 128)).astype(
        np.float32), cuda)
    g = _t(r.uniform(0.5, 1.5, 128).astype(np.float32), cuda)
    out = torch.empty(64, 128, device=cuda)
    nd = ggml.node(ggml.OP_FUSED_RMS_SILU_GATE, ggml.f32_desc(out),
                   [ggml.f32_desc(o), ggml.f32_desc(z), ggml.f32_desc(g)], [1e-6])
    assert ggml.compute_forward(nd) == 0
    ref = ops.rms_norm_silu_gate_f32(o, z, g, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("B", [2, 5])
def test_layer_decode_node(cuda, B):
    """The layer node and the layer entry, from equal states, give equal y,
    conv state and recurrent state."""
    import torch
    from leaninfer_b200 import ggml, ops, synth
    r = rng(920 + B)
    hidden, Hk, Hv, D = 1024, 4, 8, 128
    w = synth.deltanet_layer(r, hidden=hidden, n_k_heads=Hk, n_v_heads=Hv, wtype=12)
    inp = synth.deltanet_inputs(r, B, w)
    t = lambda a: _t(a, cuda)
    d = {k: t(w[k]) for k in ("w_in", "conv_w", "a_log", "dt_bias", "norm_w", "w_out")}
    layer = ops.DeltaNetLayerDecode(hidden=hidden, n_k_heads=Hk, n_v_heads=Hv, head_dim=D, **d)
    x = t((r.standard_normal((B, hidden)) * synth.DELTANET_X_SCALE).astype(np.float32))
    cs1, st1 = t(inp["conv_state"]), t(inp["state"])
    cs2, st2 = cs1.clone(), st1.clone()
    y1, y2 = torch.empty(B, hidden, device=cuda), torch.empty(B, hidden, device=cuda)
    layer.step(x, y1, cs1, st1)
    C = 2 * Hk * D + Hv * D
    NI = C + Hv * D + 2 * Hv
    srcs = [ggml.f32_desc(x), ggml.f32_desc(cs2), ggml.f32_desc(st2), ggml.quant_desc(d["w_in"], 12, hidden, NI),
            ggml.f32_desc(d["conv_w"]), ggml.f32_desc(d["a_log"]), ggml.f32_desc(d["dt_bias"]),
            ggml.f32_desc(d["norm_w"]), ggml.quant_desc(d["w_out"], 12, Hv * D, hidden), None]
    nd = ggml.node(ggml.OP_DELTANET_DECODE, ggml.f32_desc(y2), srcs, [Hk, 0, 1e-6, 1e-6, 1e-6])
    ws = torch.empty(ggml.workspace_size(nd), device=cuda, dtype=torch.uint8)
    assert ggml.compute_forward(nd, ws) == 0
    torch.cuda.synchronize()
    assert torch.equal(y1, y2) and torch.equal(cs1, cs2) and torch.equal(st1, st2)


def test_descriptors_of_views_keep_their_strides(lib):
    """f32_desc reads a tensor's real strides: a transposed view is not
    contiguous, so the dispatch refuses it rather than reading it as rows."""
    import torch
    from leaninfer_b200 import ggml
    x = torch.zeros(4096, 2).t()                     # [2, 4096] view with strides (1, 2)
    d = ggml.f32_desc(x)
    assert (d.ne[0], d.ne[1]) == (4096, 2) and (d.nb[0], d.nb[1]) == (8, 4)
    W = _fake_quant(12, 4096, 64)
    assert _run(lib, ggml.node(ggml.OP_MUL_MAT, _fake_f32([64, 2]), [W, d])) == 2002
    c = ggml.f32_desc(x.contiguous())
    assert (c.nb[0], c.nb[1]) == (4, 4 * 4096)
