"""GGUF weight loading (leaninfer_b200/gguf_file.py), CPU only: files written
by gguf-py (the format's reference implementation in this image) read back
with their metadata, tensor directory and raw blocks intact; malformed files
rejected; a DeltaNet layer and an FFN assembled from their GGUF tensors
equal the weights they were written from."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rng

gguf = pytest.importorskip("gguf")


def _write(path, tensors, meta=(), alignment=None):
    w = gguf.GGUFWriter(str(path), arch="test")
    if alignment:
        w.add_custom_alignment(alignment)
    for kind, key, val in meta:
        getattr(w, f"add_{kind}")(key, val)
    for name, arr, raw in tensors:
        w.add_tensor(name, arr, raw_dtype=raw)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


@pytest.mark.parametrize("alignment", [None, 64])
def test_directory_metadata_and_raw_blocks(tmp_path, alignment):
    from leaninfer_b200 import synth
    from leaninfer_b200.gguf_file import GGUFFile
    r = rng(31)
    q4 = synth.random_weights(r, 12, 6, 512)          # uint8 [6, 288]
    q8 = synth.random_weights(r, 8, 5, 96)            # uint8 [5, 102]
    f32 = r.standard_normal((3, 5)).astype(np.float32)
    f16 = r.standard_normal(7).astype(np.float16)
    p = tmp_path / "m.gguf"
    _write(p, [("a.q4", q4, gguf.GGMLQuantizationType.Q4_K), ("b.q8", q8, gguf.GGMLQuantizationType.Q8_0),
               ("c.f32", f32, None), ("d.f16", f16, None)],
           meta=[("uint32", "t.u32", 7), ("float32", "t.f32", 0.5), ("string", "t.s", "hello"),
                 ("array", "t.arr", [1, 2, 3]), ("bool", "t.b", True)], alignment=alignment)
    with GGUFFile(p) as g:
        assert g.version == 3
        assert g.metadata["general.architecture"] == "test"
        assert g.metadata["t.u32"] == 7 and g.metadata["t.f32"] == 0.5 and g.metadata["t.s"] == "hello"
        assert g.metadata["t.arr"] == [1, 2, 3] and g.metadata["t.b"] is True
        assert list(g.tensors) == ["a.q4", "b.q8", "c.f32", "d.f16"]
        assert g.tensors["a.q4"].ne == (512, 6) and g.tensors["a.q4"].type == 12
        assert g.tensors["b.q8"].ne == (96, 5) and g.tensors["b.q8"].type == 8
        assert g.tensors["c.f32"].ne == (5, 3) and g.tensors["c.f32"].shape == (3, 5)
        if alignment:
            assert g.data_start % alignment == 0
        assert np.array_equal(g.raw("a.q4"), q4) and np.array_equal(g.raw("b.q8"), q8)
        assert np.array_equal(g.raw("c.f32"), f32) and np.array_equal(g.raw("d.f16"), f16)
        # the directory agrees with gguf-py's own reader
        rd = gguf.GGUFReader(str(p))
        for t in rd.tensors:
            info = g.tensors[t.name]
            assert tuple(int(v) for v in t.shape) == info.ne and int(t.tensor_type) == info.type
            assert int(t.data_offset) == g.data_start + info.offset


def test_loaded_blocks_dequantize_like_gguf_py(tmp_path, oracle_mod):
    from leaninfer_b200 import synth
    from leaninfer_b200.gguf_file import GGUFFile
    r = rng(32)
    for wtype, raw in ((12, gguf.GGMLQuantizationType.Q4_K), (8, gguf.GGMLQuantizationType.Q8_0)):
        w = synth.random_weights(r, wtype, 4, 256)
        p = tmp_path / f"q{wtype}.gguf"
        _write(p, [("w", w, raw)])
        with GGUFFile(p) as g:
            got = oracle_mod.dequantize(wtype, np.ascontiguousarray(g.raw("w")), 4 * 256)
        ref = gguf.quants.dequantize(w, raw).reshape(-1)
        assert np.array_equal(got.view(np.uint32), ref.astype(np.float32).view(np.uint32))


def test_malformed_files_are_rejected(tmp_path):
    from leaninfer_b200 import synth
    from leaninfer_b200.gguf_file import GGUFError, GGUFFile
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + bytes(20))
    with pytest.raises(GGUFError):
        GGUFFile(bad)
    empty = tmp_path / "empty.gguf"
    empty.write_bytes(b"")
    with pytest.raises(GGUFError):
        GGUFFile(empty)
    p = tmp_path / "t.gguf"
    _write(p, [("w", synth.random_weights(rng(33), 12, 8, 256), gguf.GGMLQuantizationType.Q4_K)])
    data = p.read_bytes()
    cut = tmp_path / "cut.gguf"
    cut.write_bytes(data[:-100])                     # last tensor runs past the end
    with pytest.raises(GGUFError):
        GGUFFile(cut)
    head = tmp_path / "head.gguf"
    head.write_bytes(data[:30])                      # header itself truncated
    with pytest.raises(GGUFError):
        GGUFFile(head)


def test_deltanet_layer_from_gguf(tmp_path, oracle_mod):
    """A layer written as llama.cpp-style tensors (in-projection in four row
    blocks) loads back bit-identical, and the oracle's decode step from it
    equals the step from the original weights."""
    from leaninfer_b200 import synth
    from leaninfer_b200.gguf_file import DELTANET_NAMES, GGUFFile, deltanet_layer
    r = rng(34)
    hidden, Hk, Hv, D = 256, 1, 2, 128
    w = synth.deltanet_layer(r, hidden=hidden, n_k_heads=Hk, n_v_heads=Hv, head_dim=D, wtype=12)
    C = 2 * Hk * D + Hv * D
    cuts = np.cumsum([C, Hv * D, Hv])
    parts = np.split(w["w_in"], cuts)
    Q = gguf.GGMLQuantizationType.Q4_K
    il = 3
    names = [n.format(il=il) for n in DELTANET_NAMES["in_proj"]]
    tensors = [(n, part, Q) for n, part in zip(names, parts)] + [
        (DELTANET_NAMES["conv_w"].format(il=il), w["conv_w"], None),
        (DELTANET_NAMES["a_log"].format(il=il), w["a_log"], None),
        (DELTANET_NAMES["dt_bias"].format(il=il), w["dt_bias"], None),
        (DELTANET_NAMES["norm_w"].format(il=il), w["norm_w"], None),
        (DELTANET_NAMES["w_out"].format(il=il), w["w_out"], Q)]
    p = tmp_path / "layer.gguf"
    _write(p, tensors)
    with GGUFFile(p) as g:
        got = deltanet_layer(g, il, n_k_heads=Hk, n_v_heads=Hv, head_dim=D)
    for k, v in w.items():
        if isinstance(v, np.ndarray):
            assert np.array_equal(got[k], v), k
        else:
            assert got[k] == v, k
    inp = synth.deltanet_inputs(r, 2, w)
    x = (r.standard_normal((2, hidden)) * synth.DELTANET_X_SCALE).astype(np.float32)
    outs = []
    for lw in (w, got):
        L, keep = oracle_mod.make_layer(lw)
        cs, st = inp["conv_state"].copy(), inp["state"].copy()
        outs.append((oracle_mod.deltanet_layer_decode(L, keep, x, cs, st), cs, st))
    for a, b in zip(outs[0], outs[1]):
        assert np.array_equal(a, b)


def test_ffn_weights_from_gguf(tmp_path, oracle_mod):
    from leaninfer_b200 import synth
    from leaninfer_b200.gguf_file import FFN_NAMES, GGUFError, GGUFFile, ffn_weights
    r = rng(35)
    K, N = 256, 512
    Wg, Wu, Wd = (synth.random_weights(r, 8, N, K), synth.random_weights(r, 8, N, K),
                  synth.random_weights(r, 8, K, N))
    Q = gguf.GGMLQuantizationType.Q8_0
    p = tmp_path / "ffn.gguf"
    _write(p, [(FFN_NAMES["gate"].format(il=0), Wg, Q), (FFN_NAMES["up"].format(il=0), Wu, Q),
               (FFN_NAMES["down"].format(il=0), Wd, Q), (FFN_NAMES["down"].format(il=1), Wg, Q),
               (FFN_NAMES["gate"].format(il=1), Wg, Q), (FFN_NAMES["up"].format(il=1), Wu, Q)])
    x = r.standard_normal((2, K)).astype(np.float32)
    gamma = r.uniform(0.5, 1.5, K).astype(np.float32)
    with GGUFFile(p) as g:
        f = ffn_weights(g, 0)
        assert (f["wtype"], f["K"], f["N"]) == (8, K, N)
        y = oracle_mod.ffn(8, x, gamma, np.ascontiguousarray(f["Wg"]), np.ascontiguousarray(f["Wu"]),
                           np.ascontiguousarray(f["Wd"]), N)
        with pytest.raises(GGUFError):
            ffn_weights(g, 1)                       # down written with the gate's shape
    assert np.array_equal(y, oracle_mod.ffn(8, x, gamma, Wg, Wu, Wd, N))


def test_qkv_weights_from_gguf(tmp_path, oracle_mod):
    from leaninfer_b200 import synth
    from leaninfer_b200.gguf_file import QKV_NAMES, GGUFError, GGUFFile, qkv_weights
    r = rng(36)
    K = 512
    Ws = {k: synth.random_weights(r, 8, n, K) for k, n in (("q", 512), ("k", 128), ("v", 128))}
    gamma = r.uniform(0.5, 1.5, K).astype(np.float32)
    Q = gguf.GGMLQuantizationType.Q8_0
    p = tmp_path / "qkv.gguf"
    _write(p, [(QKV_NAMES[k].format(il=2), Ws[k], Q) for k in ("q", "k", "v")] +
           [(QKV_NAMES["norm"].format(il=2), gamma, None), (QKV_NAMES["norm"].format(il=5), gamma[:256], None)] +
           [(QKV_NAMES[k].format(il=5), Ws[k], Q) for k in ("q", "k", "v")] +
           [(QKV_NAMES[k].format(il=6), Ws[k], Q) for k in ("q", "k", "v")] +
           [(QKV_NAMES["norm"].format(il=6), synth.random_weights(r, 8, 1, K).reshape(-1), Q),
            (QKV_NAMES["norm"].format(il=7), gamma.astype(np.float16), None)] +
           [(QKV_NAMES[k].format(il=7), Ws[k], Q) for k in ("q", "k", "v")])
    x = r.standard_normal((1, K)).astype(np.float32)
    with GGUFFile(p) as g:
        f = qkv_weights(g, 2)
        assert (f["wtype"], f["K"], f["Nq"], f["Nk"], f["Nv"]) == (8, K, 512, 128, 128)
        assert np.array_equal(f["gamma"], gamma)
        for k, n in (("q", 512), ("k", 128), ("v", 128)):
            W = f["W" + k]
            assert np.array_equal(oracle_mod.rms_norm_matmul(8, x, f["gamma"], np.ascontiguousarray(W), n),
                                  oracle_mod.rms_norm_matmul(8, x, gamma, Ws[k], n))
        with pytest.raises(GGUFError):
            qkv_weights(g, 5)                       # norm weight of the wrong width
        with pytest.raises(GGUFError):
            qkv_weights(g, 6)                       # a quantized norm weight (K values as Q8_0 blocks)
        f16 = qkv_weights(g, 7)                     # an F16 norm weight is widened exactly
        assert np.array_equal(f16["gamma"], gamma.astype(np.float16).astype(np.float32))
