"""GGUF weight loading: the tensor directory of a GGUF file (v2/v3) and raw
views of its tensors, so real Q4_K / Q8_0 checkpoints feed the kernels the
blocks they hold (no requantization, no dequantization).

File layout (little endian): magic "GGUF", u32 version, u64 tensor count,
u64 metadata count; metadata entries (string key, u32 value type, value);
tensor infos (string name, u32 n_dims, u64 ne[n_dims] innermost first, u32
ggml type, u64 offset from the data section); the data section starts at
the next multiple of `general.alignment` (32 when absent). Strings are a
u64 length and UTF-8 bytes. The reference reads the same directory
(profiles/profiler.py:110-139) for its router analysis; here the file is
memory-mapped and every tensor is checked to lie inside the file.
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

MAGIC = b"GGUF"
# metadata value types
_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
_STRING, _ARRAY = 8, 9
# ggml types this loader hands out: (values per block, bytes per block)
TYPE_BLOCKS = {0: (1, 4), 1: (1, 2), 8: (32, 34), 12: (256, 144), 30: (1, 2)}
TYPE_NAMES = {0: "F32", 1: "F16", 8: "Q8_0", 12: "Q4_K", 30: "BF16"}


class GGUFError(ValueError):
    pass


@dataclass(frozen=True)
class TensorInfo:
    name: str
    ne: tuple[int, ...]     # elements per dimension, innermost first (ggml order)
    type: int               # ggml type id
    offset: int             # byte offset inside the data section
    nbytes: int

    @property
    def shape(self) -> tuple[int, ...]:
        """numpy (row-major) shape: ne reversed."""
        return tuple(reversed(self.ne))

    @property
    def row_bytes(self) -> int:
        blk, size = TYPE_BLOCKS[self.type]
        return self.ne[0] // blk * size


class GGUFFile:
    """A GGUF file opened read-only: `metadata` (key -> value), `tensors`
    (name -> TensorInfo in file order) and `raw(name)` views."""

    def __init__(self, path: str | Path):
        self.path = Path(path)
        self._f = open(self.path, "rb")
        try:
            self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        except ValueError as e:   # empty file
            self._f.close()
            raise GGUFError(f"{self.path}: not a GGUF file") from e
        self._pos = 0
        try:
            self._parse()
        except (struct.error, UnicodeDecodeError, IndexError) as e:
            self.close()
            raise GGUFError(f"{self.path}: truncated or malformed header ({e})") from e
        except GGUFError:
            self.close()
            raise

    # ---- primitive reads ----
    def _take(self, n: int) -> bytes:
        if self._pos + n > len(self._mm):
            raise GGUFError(f"{self.path}: header runs past the end of the file")
        b = self._mm[self._pos:self._pos + n]
        self._pos += n
        return b

    def _u32(self) -> int:
        return struct.unpack("<I", self._take(4))[0]

    def _u64(self) -> int:
        return struct.unpack("<Q", self._take(8))[0]

    def _str(self) -> str:
        return self._take(self._u64()).decode("utf-8")

    def _value(self, vtype: int, depth: int = 0):
        if vtype in _SCALAR:
            fmt = _SCALAR[vtype]
            return struct.unpack(fmt, self._take(struct.calcsize(fmt)))[0]
        if vtype == _STRING:
            return self._str()
        if vtype == _ARRAY:
            if depth > 4:
                raise GGUFError(f"{self.path}: metadata arrays nested too deep")
            etype, n = self._u32(), self._u64()
            return [self._value(etype, depth + 1) for _ in range(n)]
        raise GGUFError(f"{self.path}: unknown metadata value type {vtype}")

    # ---- header ----
    def _parse(self):
        if self._take(4) != MAGIC:
            raise GGUFError(f"{self.path}: not a GGUF file")
        self.version = self._u32()
        if self.version not in (2, 3):
            raise GGUFError(f"{self.path}: GGUF version {self.version} is not supported (2 and 3 are)")
        n_tensors, n_kv = self._u64(), self._u64()
        self.metadata: dict = {}
        for _ in range(n_kv):
            key = self._str()
            self.metadata[key] = self._value(self._u32())
        infos = []
        for _ in range(n_tensors):
            name = self._str()
            nd = self._u32()
            if nd < 1 or nd > 4:
                raise GGUFError(f"{self.path}: tensor {name} has {nd} dimensions")
            ne = tuple(self._u64() for _ in range(nd))
            t, off = self._u32(), self._u64()
            infos.append((name, ne, t, off))
        align = int(self.metadata.get("general.alignment", 32))
        if align <= 0 or align & (align - 1):
            raise GGUFError(f"{self.path}: alignment {align} is not a power of two")
        self.data_start = (self._pos + align - 1) // align * align
        self.tensors: dict[str, TensorInfo] = {}
        for name, ne, t, off in infos:
            nbytes = None
            if t in TYPE_BLOCKS:
                blk, size = TYPE_BLOCKS[t]
                if ne[0] % blk:
                    raise GGUFError(f"{self.path}: tensor {name}: ne[0] = {ne[0]} is not a multiple of {blk}")
                nbytes = int(np.prod(ne, dtype=np.int64)) // blk * size
            if nbytes is not None and self.data_start + off + nbytes > len(self._mm):
                raise GGUFError(f"{self.path}: tensor {name} runs past the end of the file")
            self.tensors[name] = TensorInfo(name, ne, t, off, nbytes if nbytes is not None else -1)

    # ---- tensors ----
    def raw(self, name: str) -> np.ndarray:
        """Read-only view of a tensor: quantized types as uint8 [rows,
        row_bytes] (rows = product of ne[1:]), F32 / F16 as float32 /
        float16 arrays of the numpy shape, BF16 as uint16."""
        info = self.tensors.get(name)
        if info is None:
            raise KeyError(name)
        if info.type not in TYPE_BLOCKS:
            raise GGUFError(f"{self.path}: tensor {name} has ggml type {info.type}, which this loader does not map")
        buf = np.frombuffer(self._mm, dtype=np.uint8, count=info.nbytes, offset=self.data_start + info.offset)
        if info.type in (8, 12):
            return buf.reshape(-1, info.row_bytes)
        dt = {0: np.float32, 1: np.float16, 30: np.uint16}[info.type]
        return buf.view(dt).reshape(info.shape)

    def close(self):
        if getattr(self, "_mm", None) is not None:
            try:
                self._mm.close()
            except BufferError:   # views still alive: the map closes with them
                pass
            self._mm = None
        if not self._f.closed:
            self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


# In-projection row blocks of a Gated DeltaNet layer, in the order the layer
# decode wants (q | k | v | z | beta | alpha), and the other tensors. The
# names follow llama.cpp's ssm_* convention; converters differ, so callers
# pass their own map.
DELTANET_NAMES = {
    "in_proj": ["blk.{il}.attn_qkv.weight", "blk.{il}.attn_gate.weight", "blk.{il}.ssm_beta.weight",
                "blk.{il}.ssm_alpha.weight"],
    "conv_w": "blk.{il}.ssm_conv1d.weight",
    "a_log": "blk.{il}.ssm_a",
    "dt_bias": "blk.{il}.ssm_dt.bias",
    "norm_w": "blk.{il}.ssm_norm.weight",
    "w_out": "blk.{il}.ssm_out.weight",
}


def deltanet_layer(g: GGUFFile, il: int, *, n_k_heads: int, n_v_heads: int, head_dim: int = 128,
                   names: dict | None = None) -> dict:
    """The weights of DeltaNet layer `il` in the form the layer decode takes
    (the dict leaninfer_b200.synth.deltanet_layer returns): the in-projection
    parts' quantized rows stacked in order (rows are independent, so the
    blocks are copied, not converted), conv weights [C, 4], a_log, dt_bias,
    gated-norm gamma, out-projection rows. All quantized parts must share
    one type (Q4_K or Q8_0)."""
    nm = names or DELTANET_NAMES
    D, Hk, Hv = head_dim, n_k_heads, n_v_heads
    C = 2 * Hk * D + Hv * D
    NI = C + Hv * D + 2 * Hv
    parts = [g.tensors[n.format(il=il)] for n in nm["in_proj"]]
    wtype = parts[0].type
    if wtype not in (8, 12) or any(p.type != wtype for p in parts):
        raise GGUFError(f"layer {il}: in-projection parts must share one quantized type (Q4_K or Q8_0)")
    hidden = parts[0].ne[0]
    if any(p.ne[0] != hidden for p in parts):
        raise GGUFError(f"layer {il}: in-projection parts disagree on the input width")
    w_in = np.concatenate([g.raw(p.name) for p in parts], axis=0)
    if w_in.shape[0] != NI:
        raise GGUFError(f"layer {il}: in-projection has {w_in.shape[0]} rows, the heads need {NI}")
    out = g.tensors[nm["w_out"].format(il=il)]
    if out.type != wtype or out.ne != (Hv * D, hidden):
        raise GGUFError(f"layer {il}: out-projection is not {TYPE_NAMES.get(wtype)} [{Hv * D}, {hidden}]")

    def f32(key, shape):
        a = np.asarray(g.raw(nm[key].format(il=il)), dtype=np.float32).reshape(shape)
        return np.ascontiguousarray(a)
    return dict(hidden=hidden, n_k_heads=Hk, n_v_heads=Hv, head_dim=D, wtype=wtype,
                w_in=np.ascontiguousarray(w_in), conv_w=f32("conv_w", (C, 4)), a_log=f32("a_log", (Hv,)),
                dt_bias=f32("dt_bias", (Hv,)), norm_w=f32("norm_w", (D,)),
                w_out=np.ascontiguousarray(g.raw(out.name)))


FFN_NAMES = {"gate": "blk.{il}.ffn_gate.weight", "up": "blk.{il}.ffn_up.weight", "down": "blk.{il}.ffn_down.weight"}


def ffn_weights(g: GGUFFile, il: int, names: dict | None = None) -> dict:
    """The SwiGLU FFN of layer `il` for the FFN entries: Wg, Wu [N rows of K]
    and Wd [K rows of N] as the file's quantized rows, with K (model width),
    N (inner width) and the shared weight type."""
    nm = names or FFN_NAMES
    tg, tu, td = (g.tensors[nm[k].format(il=il)] for k in ("gate", "up", "down"))
    wtype = tg.type
    if wtype not in (8, 12) or tu.type != wtype or td.type != wtype:
        raise GGUFError(f"layer {il}: FFN matrices must share one quantized type (Q4_K or Q8_0)")
    K, N = tg.ne[0], tg.ne[1]
    if tu.ne != (K, N) or td.ne != (N, K):
        raise GGUFError(f"layer {il}: FFN shapes gate {tg.ne}, up {tu.ne}, down {td.ne} do not match")
    return dict(wtype=wtype, K=K, N=N, Wg=g.raw(tg.name), Wu=g.raw(tu.name), Wd=g.raw(td.name))


QKV_NAMES = {"q": "blk.{il}.attn_q.weight", "k": "blk.{il}.attn_k.weight", "v": "blk.{il}.attn_v.weight",
             "norm": "blk.{il}.attn_norm.weight"}


def qkv_weights(g: GGUFFile, il: int, names: dict | None = None) -> dict:
    """The attention input projections of layer `il` for the fused RMSNorm +
    Q/K/V entry: Wq, Wk, Wv as the file's quantized rows (one shared type and
    input width K), their row counts Nq, Nk, Nv, and the RMSNorm weight."""
    nm = names or QKV_NAMES
    tq, tk, tv = (g.tensors[nm[k].format(il=il)] for k in ("q", "k", "v"))
    wtype, K = tq.type, tq.ne[0]
    if wtype not in (8, 12) or tk.type != wtype or tv.type != wtype:
        raise GGUFError(f"layer {il}: Q/K/V must share one quantized type (Q4_K or Q8_0)")
    if any(len(t.ne) != 2 or t.ne[0] != K for t in (tq, tk, tv)):
        raise GGUFError(f"layer {il}: Q/K/V disagree on the input width")
    tn = g.tensors[nm["norm"].format(il=il)]
    if tn.type == 0:                    # F32
        gamma = np.asarray(g.raw(tn.name), dtype=np.float32).reshape(-1)
    elif tn.type == 1:                  # F16, widened exactly
        gamma = np.asarray(g.raw(tn.name)).astype(np.float32).reshape(-1)
    else:
        raise GGUFError(f"layer {il}: the norm weight has ggml type {tn.type}; F32 or F16 expected")
    if gamma.shape[0] != K:
        raise GGUFError(f"layer {il}: the norm weight has {gamma.shape[0]} values, the projections take {K}")
    return dict(wtype=wtype, K=K, Nq=tq.ne[1], Nk=tk.ne[1], Nv=tv.ne[1], Wq=g.raw(tq.name), Wk=g.raw(tk.name),
                Wv=g.raw(tv.name), gamma=np.ascontiguousarray(gamma))
