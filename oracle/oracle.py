"""ctypes wrapper of the CPU oracle (liboracle.so) and of the reference's own
sources built into oracle/_ref/.

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg use it as the checker. It is never the thing measured on the
GPU and nothing in leaninfer_b200/ imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, c_float, c_int, c_int64, c_size_t, c_uint16, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_BENCH = HERE / "_ref" / "libliref_bench.so"
REF_GPU = HERE / "_ref" / "libliref_gpu.so"
# The reference checkout, only where it is mounted (never on the GPU box):
# its sources are compiled where they lie into _ref/.
REF_SRC = Path(os.environ["LEANINFER_REF_SRC"]) if os.environ.get("LEANINFER_REF_SRC") else None

Q8_0, Q4_K = 8, 12


class Layer(ctypes.Structure):
    _fields_ = [
        ("hidden", c_int), ("n_k_heads", c_int), ("n_v_heads", c_int), ("head_dim", c_int),
        ("conv_kernel", c_int), ("repeat_type", c_int), ("w_in_type", c_int), ("w_out_type", c_int),
        ("in_norm_eps", c_float), ("norm_eps", c_float), ("l2_eps", c_float),
        ("in_norm_w", c_void_p), ("w_in", c_void_p), ("conv_w", c_void_p), ("a_log", c_void_p),
        ("dt_bias", c_void_p), ("norm_w", c_void_p), ("w_out", c_void_p),
    ]


class AttnLayer(ctypes.Structure):
    _fields_ = [
        ("hidden", c_int), ("n_q_heads", c_int), ("n_kv_heads", c_int), ("head_dim", c_int), ("rope_dim", c_int),
        ("w_in_type", c_int), ("w_out_type", c_int),
        ("rope_theta", c_float), ("in_norm_eps", c_float), ("qk_norm_eps", c_float),
        ("in_norm_w", c_void_p), ("w_in", c_void_p), ("q_norm_w", c_void_p), ("k_norm_w", c_void_p),
        ("w_out", c_void_p),
    ]


_lib = None
NATIVE = HERE / "_native" / "liboracle_native.so"


def use_native() -> bool:
    """Build the oracle with -march=native for the host it runs on (the CPU
    baseline legs of bench.py, on the GPU box) and load that copy instead of
    the portable one; False (and the portable copy stays) if the build fails.
    Call before the first use of lib()."""
    global _lib
    if _lib is not None:
        return False
    r = subprocess.run(["make", "-s", "-C", str(HERE), "native"], capture_output=True, text=True)
    if r.returncode != 0 or not NATIVE.exists():
        return False
    _load(NATIVE)
    return True


def build(with_ref: bool | None = None) -> None:
    """make liboracle.so; with_ref (default: when LEANINFER_REF_SRC names an
    existing reference checkout) also builds the reference's sources into
    _ref/."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    if with_ref is None:
        with_ref = REF_SRC is not None and REF_SRC.is_dir()
    if with_ref:
        if REF_SRC is None:
            raise RuntimeError("LEANINFER_REF_SRC is not set: no reference checkout to build _ref/ from")
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF={REF_SRC}"], check=True,
                       stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)


def lib() -> ctypes.CDLL:
    if _lib is None:
        if not LIB.exists() or LIB.stat().st_mtime < (HERE / "li_oracle.c").stat().st_mtime:
            build(with_ref=False)
        _load(LIB)
    return _lib


def _load(path: Path) -> None:
    global _lib
    L = ctypes.CDLL(str(path))
    L.lio_dequantize.argtypes = [c_int, c_void_p, c_void_p, c_int64]
    L.lio_rms_norm_matmul.argtypes = [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                      c_float]
    L.lio_rms_norm_matmul_q8act.argtypes = [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                            c_int, c_float]
    L.lio_rms_norm_swiglu.argtypes = [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                      c_int, c_int, c_float, c_int]
    L.lio_ffn.argtypes = [c_int] + [c_void_p] * 6 + [c_int, c_int, c_int, c_float]
    L.lio_silu_gate.argtypes = [c_void_p] * 4 + [c_int, c_int, c_float]
    L.lio_silu_gate.restype = None
    L.lio_deltanet_recurrent.argtypes = [c_void_p] * 10 + [c_int64] * 4 + [c_int, c_int64, c_int64,
                                                                            c_size_t, c_size_t, c_size_t]
    L.lio_deltanet_taps_per_seq.argtypes = [POINTER(Layer)]
    L.lio_deltanet_taps_per_seq.restype = c_size_t
    L.lio_deltanet_layer_decode.argtypes = [POINTER(Layer), c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                            c_void_p]
    L.lio_deltanet_layer_decode_q8act.argtypes = [POINTER(Layer), c_void_p, c_void_p, c_void_p, c_void_p, c_int]
    L.lio_gdr_prefill.argtypes = [c_void_p] * 7 + [c_int, c_int, c_int, c_int, c_float]
    L.lio_fp16_to_fp32.argtypes = [c_uint16]
    L.lio_fp16_to_fp32.restype = c_float
    L.lio_fp32_to_fp16.argtypes = [c_float]
    L.lio_fp32_to_fp16.restype = c_uint16
    L.lio_attn_layer_decode.argtypes = [POINTER(AttnLayer)] + [c_void_p] * 5 + [c_int, c_int]
    L.lio_num_threads.restype = c_int
    _lib = L


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def num_threads() -> int:
    return int(lib().lio_num_threads())


def dequantize(wtype: int, blocks: np.ndarray, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    assert lib().lio_dequantize(wtype, _ptr(np.ascontiguousarray(blocks)), _ptr(out), n) == 0
    return out


def rms_norm_matmul(wtype, x, gamma, W, N, eps=1e-6):
    x = _f32(np.atleast_2d(x))
    n_rows, K = x.shape
    out = np.empty((n_rows, N), np.float32)
    g = None if gamma is None else _f32(gamma)
    assert lib().lio_rms_norm_matmul(wtype, _ptr(x), _ptr(g), _ptr(np.ascontiguousarray(W)), _ptr(out), K, N,
                                     n_rows, eps) == 0
    return out


def rms_norm_matmul_q8act(wtype, x, gamma, W, N, eps=1e-6):
    """ggml-style quantized-activation matmul (unpinned; see li_oracle.h)."""
    x = _f32(np.atleast_2d(x))
    n_rows, K = x.shape
    out = np.empty((n_rows, N), np.float32)
    g = None if gamma is None else _f32(gamma)
    assert lib().lio_rms_norm_matmul_q8act(wtype, _ptr(x), _ptr(g), _ptr(np.ascontiguousarray(W)), _ptr(out), K,
                                           N, n_rows, eps) == 0
    return out


def rms_norm_swiglu(wtype, x, gamma, Wg, Wu, N, eps=1e-6, round_xn_f16=False):
    x = _f32(np.atleast_2d(x))
    n_rows, K = x.shape
    out = np.empty((n_rows, N), np.float32)
    assert lib().lio_rms_norm_swiglu(wtype, _ptr(x), _ptr(_f32(gamma)), _ptr(np.ascontiguousarray(Wg)),
                                     _ptr(np.ascontiguousarray(Wu)), _ptr(out), K, N, n_rows, eps,
                                     int(round_xn_f16)) == 0
    return out


def ffn(wtype, x, gamma, Wg, Wu, Wd, N, eps=1e-6):
    x = _f32(np.atleast_2d(x))
    n_rows, K = x.shape
    out = np.empty((n_rows, K), np.float32)
    assert lib().lio_ffn(wtype, _ptr(x), _ptr(_f32(gamma)), _ptr(np.ascontiguousarray(Wg)),
                         _ptr(np.ascontiguousarray(Wu)), _ptr(np.ascontiguousarray(Wd)), _ptr(out), K, N,
                         n_rows, eps) == 0
    return out


def silu_gate(o, z, gamma, eps=1e-6):
    o, z = _f32(o), _f32(z)
    K = o.shape[-1]
    out = np.empty_like(o)
    lib().lio_silu_gate(_ptr(o), _ptr(z), _ptr(_f32(gamma)), _ptr(out), K, o.size // K, eps)
    return out


def deltanet_recurrent(q, k, v, g, beta, state_in, *, D, n_tokens, n_heads, gqa, repeat_type, n_seqs,
                       vnb1, vnb2, vnb3, W_out=None, hidden=0):
    """Reference-layout recurrence. Returns (out, state_out, proj_out or None)."""
    out = np.empty(n_seqs * n_tokens * n_heads * D, np.float32)
    st = np.empty(np.asarray(state_in).size, np.float32)
    proj = np.empty(hidden * n_tokens, np.float32) if W_out is not None else None
    rc = lib().lio_deltanet_recurrent(_ptr(_f32(q)), _ptr(_f32(k)), _ptr(_f32(v)), _ptr(_f32(g)),
                                      _ptr(_f32(beta)), _ptr(_f32(state_in)), _ptr(out), _ptr(st),
                                      _ptr(None if W_out is None else _f32(W_out)), _ptr(proj), D, n_tokens,
                                      n_heads, gqa, repeat_type, n_seqs, hidden, vnb1, vnb2, vnb3)
    assert rc == 0
    return out, st, proj


def make_layer(w: dict, in_norm_w=None, norm_eps=1e-6, l2_eps=1e-6, in_norm_eps=1e-6, repeat_type=0):
    keep = dict(w)
    for name in ("conv_w", "a_log", "dt_bias", "norm_w"):
        keep[name] = _f32(w[name])
    keep["w_in"] = np.ascontiguousarray(w["w_in"])
    keep["w_out"] = np.ascontiguousarray(w["w_out"])
    keep["in_norm_w"] = None if in_norm_w is None else _f32(in_norm_w)
    L = Layer(hidden=w["hidden"], n_k_heads=w["n_k_heads"], n_v_heads=w["n_v_heads"], head_dim=w["head_dim"],
              conv_kernel=4, repeat_type=repeat_type, w_in_type=w["wtype"], w_out_type=w["wtype"],
              in_norm_eps=in_norm_eps, norm_eps=norm_eps, l2_eps=l2_eps,
              in_norm_w=_ptr(keep["in_norm_w"]), w_in=_ptr(keep["w_in"]), conv_w=_ptr(keep["conv_w"]),
              a_log=_ptr(keep["a_log"]), dt_bias=_ptr(keep["dt_bias"]), norm_w=_ptr(keep["norm_w"]),
              w_out=_ptr(keep["w_out"]))
    return L, keep


def deltanet_layer_decode(layer, keep, x, conv_state, state, with_taps=False):
    """One step; conv_state and state (float32 numpy) are updated in place."""
    x = _f32(np.atleast_2d(x))
    n = x.shape[0]
    y = np.empty((n, layer.hidden), np.float32)
    taps = None
    if with_taps:
        taps = np.empty((n, lib().lio_deltanet_taps_per_seq(ctypes.byref(layer))), np.float32)
    assert conv_state.dtype == np.float32 and conv_state.flags["C_CONTIGUOUS"]
    assert state.dtype == np.float32 and state.flags["C_CONTIGUOUS"]
    assert lib().lio_deltanet_layer_decode(ctypes.byref(layer), _ptr(x), _ptr(y), _ptr(conv_state),
                                           _ptr(state), n, _ptr(taps)) == 0
    return (y, taps) if with_taps else y


def fp32_to_fp16_bits(f: float) -> int:
    return int(lib().lio_fp32_to_fp16(float(f)))


def make_attn_layer(w: dict):
    """w: synth.attn_layer's dict (weights as numpy, shapes and eps)."""
    keep = {k: (_f32(v) if isinstance(v, np.ndarray) and v.dtype != np.uint8 else
                (np.ascontiguousarray(v) if isinstance(v, np.ndarray) else v)) for k, v in w.items()}
    L = AttnLayer(hidden=w["hidden"], n_q_heads=w["n_q_heads"], n_kv_heads=w["n_kv_heads"], head_dim=w["head_dim"],
                  rope_dim=w["rope_dim"], w_in_type=w["wtype"], w_out_type=w["wtype"], rope_theta=w["rope_theta"],
                  in_norm_eps=w["eps"], qk_norm_eps=w["eps"],
                  in_norm_w=_ptr(keep.get("in_norm_w")), w_in=_ptr(keep["w_in"]),
                  q_norm_w=_ptr(keep.get("q_norm_w")), k_norm_w=_ptr(keep.get("k_norm_w")),
                  w_out=_ptr(keep["w_out"]))
    return L, keep


def attn_layer_decode(layer, keep, x, k_cache, v_cache, pos):
    """One step; the fp16 caches (uint16 [n, max_ctx, Hkv, D]) get the new
    token's k, v at pos[s]."""
    x = _f32(np.atleast_2d(x))
    n = x.shape[0]
    y = np.empty((n, layer.hidden), np.float32)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    assert k_cache.dtype == np.uint16 and v_cache.dtype == np.uint16
    assert k_cache.flags["C_CONTIGUOUS"] and v_cache.flags["C_CONTIGUOUS"]
    max_ctx = k_cache.shape[1]
    assert lib().lio_attn_layer_decode(ctypes.byref(layer), _ptr(x), _ptr(y), _ptr(k_cache), _ptr(v_cache),
                                       _ptr(pos), n, max_ctx) == 0
    return y


def deltanet_layer_decode_q8act(layer, keep, x, conv_state, state):
    """One step with ggml-style quantized-activation projections (the CPU
    baseline's arithmetic; unpinned); states updated in place."""
    x = _f32(np.atleast_2d(x))
    n = x.shape[0]
    y = np.empty((n, layer.hidden), np.float32)
    assert lib().lio_deltanet_layer_decode_q8act(ctypes.byref(layer), _ptr(x), _ptr(y), _ptr(conv_state),
                                                 _ptr(state), n) == 0
    return y


def ffn_q8act(wtype, x, gamma, Wg, Wu, Wd, N, eps=1e-6):
    """The SwiGLU FFN with ggml-style quantized-activation matmuls (the CPU
    baseline's arithmetic; unpinned)."""
    g = rms_norm_matmul_q8act(wtype, x, gamma, Wg, N, eps)
    u = rms_norm_matmul_q8act(wtype, x, gamma, Wu, N, eps)
    h = (g / (1.0 + np.exp(-g.astype(np.float64))) * u).astype(np.float32)
    return rms_norm_matmul_q8act(wtype, h, None, Wd, np.atleast_2d(x).shape[1])


def gdr_prefill(q_bf16, k_bf16, v_bf16, g, beta, state, scale):
    """q, k [T, Hk, D]; v [T, Hv, D] as uint16 bf16 bits; state updated in place."""
    T, Hk, D = q_bf16.shape
    Hv = v_bf16.shape[1]
    o = np.empty((T, Hv, D), np.float32)
    assert lib().lio_gdr_prefill(_ptr(np.ascontiguousarray(q_bf16)), _ptr(np.ascontiguousarray(k_bf16)),
                                 _ptr(np.ascontiguousarray(v_bf16)), _ptr(_f32(g)), _ptr(_f32(beta)),
                                 _ptr(state), _ptr(o), T, Hk, Hv, D, scale) == 0
    return o


# ---------------------------------------------------------------------------
# The reference's own CPU function (cuda/benchmark_fused.cu:99-121), built by
# `make ref` from the reference source tree.
# ---------------------------------------------------------------------------
def ref_cpu_rms_norm_swiglu(x, gamma, Wg, Wu, eps):
    if not REF_BENCH.exists():
        raise FileNotFoundError(f"{REF_BENCH} not built (make -C oracle ref)")
    L = ctypes.CDLL(str(REF_BENCH))
    fn = L["_Z19cpu_rms_norm_swigluPKfS0_S0_S0_Pfiif"]
    fn.argtypes = [c_void_p] * 5 + [c_int, c_int, c_float]
    fn.restype = None
    x, gamma, Wg, Wu = _f32(x), _f32(gamma), _f32(Wg), _f32(Wu)
    N, K = Wg.shape
    out = np.empty(N, np.float32)
    fn(_ptr(x), _ptr(gamma), _ptr(Wg), _ptr(Wu), _ptr(out), K, N, eps)
    return out
