"""Seeded synthetic inputs in raw ggml block layouts (numpy, host side).

Used by the benchmark and the tests to build random-code quantized weights
and activations with the value distributions of the benchmark workloads:

* Q8_0 rows: fp16 scale d ~ U(1e-3, 1e-2) and int8 codes uniform on [-127, 127].
* Q4_K rows: fp16 d and dmin ~ U(1e-3, 1e-2), 12 uniformly random scale bytes
  (so every 6-bit scale and min is uniform on 0..63) and 128 uniformly random
  nibble bytes (every code uniform on 0..15).

All generators take a ``numpy.random.Generator`` (PCG64) so a seed fixes
every byte.
"""
from __future__ import annotations

import numpy as np

Q8_0, Q4_K = 8, 12
BLOCK = {Q8_0: (32, 34), Q4_K: (256, 144)}


def row_bytes(wtype: int, k: int) -> int:
    bs, tb = BLOCK[wtype]
    if k % bs:
        raise ValueError(f"K={k} is not a multiple of the block size {bs}")
    return k // bs * tb


def _fp16_bytes(vals: np.ndarray) -> np.ndarray:
    return vals.astype(np.float16).view(np.uint8).reshape(*vals.shape, 2)


def random_q8_0(rng: np.random.Generator, n: int, k: int) -> np.ndarray:
    """[n, k/32*34] uint8: n rows of Q8_0 blocks."""
    nb = k // 32
    d = rng.uniform(1e-3, 1e-2, size=(n, nb))
    qs = rng.integers(-127, 128, size=(n, nb, 32), dtype=np.int16).astype(np.int8)
    blocks = np.concatenate([_fp16_bytes(d), qs.view(np.uint8)], axis=2)
    return np.ascontiguousarray(blocks.reshape(n, nb * 34))


def random_q4_k(rng: np.random.Generator, n: int, k: int) -> np.ndarray:
    """[n, k/256*144] uint8: n rows of Q4_K super-blocks."""
    nb = k // 256
    d = rng.uniform(1e-3, 1e-2, size=(n, nb))
    dmin = rng.uniform(1e-3, 1e-2, size=(n, nb))
    scales = rng.integers(0, 256, size=(n, nb, 12), dtype=np.int16).astype(np.uint8)
    qs = rng.integers(0, 256, size=(n, nb, 128), dtype=np.int16).astype(np.uint8)
    blocks = np.concatenate([_fp16_bytes(d), _fp16_bytes(dmin), scales, qs], axis=2)
    return np.ascontiguousarray(blocks.reshape(n, nb * 144))


def random_weights(rng: np.random.Generator, wtype: int, n: int, k: int) -> np.ndarray:
    return random_q8_0(rng, n, k) if wtype == Q8_0 else random_q4_k(rng, n, k)


def deltanet_layer(rng: np.random.Generator, *, hidden=4096, n_k_heads=16, n_v_heads=32,
                   head_dim=128, wtype=Q4_K) -> dict:
    """Weights of one Gated DeltaNet layer (numpy). In-projection rows:
    q | k | v | z | beta | alpha; conv weights N(0, 0.1); a_log N(0, 0.5);
    dt_bias 0; gated-norm gamma U(0.5, 1.5); out-projection [hidden, Hv*D]."""
    D, Hk, Hv = head_dim, n_k_heads, n_v_heads
    C = 2 * Hk * D + Hv * D
    NI = C + Hv * D + 2 * Hv
    return dict(
        hidden=hidden, n_k_heads=Hk, n_v_heads=Hv, head_dim=D, wtype=wtype,
        w_in=random_weights(rng, wtype, NI, hidden),
        conv_w=rng.normal(0.0, 0.1, size=(C, 4)).astype(np.float32),
        a_log=rng.normal(0.0, 0.5, size=Hv).astype(np.float32),
        dt_bias=np.zeros(Hv, np.float32),
        norm_w=rng.uniform(0.5, 1.5, size=D).astype(np.float32),
        w_out=random_weights(rng, wtype, hidden, Hv * D),
    )


# Activation scale of the DeltaNet decode workload: with the random-code
# Q4_K weights above a row dot with x ~ N(0, 1) has a standard deviation of
# about 118, so x is drawn as N(0, 1)/128 to put the projected beta/alpha
# inputs near N(0, 1) (beta = sigmoid(N(0,1)), decay exp(-softplus(N(0,1)) *
# exp(a_log))) as the workload specifies.
DELTANET_X_SCALE = 1.0 / 128.0


def deltanet_inputs(rng: np.random.Generator, n_seqs: int, layer: dict) -> dict:
    D, Hk, Hv = layer["head_dim"], layer["n_k_heads"], layer["n_v_heads"]
    C = 2 * Hk * D + Hv * D
    return dict(
        x=(rng.standard_normal((n_seqs, layer["hidden"])) * DELTANET_X_SCALE).astype(np.float32),
        conv_state=np.zeros((n_seqs, C, 3), np.float32),
        state=rng.normal(0.0, 0.02, size=(n_seqs, Hv, D, D)).astype(np.float32),
    )


def attn_layer(rng: np.random.Generator, *, hidden=5120, n_q_heads=40, n_kv_heads=8, head_dim=128,
               rope_dim=64, rope_theta=1e7, wtype=Q4_K) -> dict:
    """Weights of one gated attention layer (numpy). In-projection rows:
    q | gate | k | v; out-projection [hidden, Hq*D]. The input RMSNorm weight
    is U(0.5, 1.5)/128, which puts a random-code Q4_K row dot of the
    normalised x near N(0, 1) (so the sigmoid gates stay informative); the
    per-head q / k norm weights are U(0.5, 1.5)."""
    D, Hq, Hkv = head_dim, n_q_heads, n_kv_heads
    NP = 2 * Hq * D + 2 * Hkv * D
    return dict(
        hidden=hidden, n_q_heads=Hq, n_kv_heads=Hkv, head_dim=D, rope_dim=rope_dim, rope_theta=rope_theta,
        wtype=wtype, eps=1e-6,
        w_in=random_weights(rng, wtype, NP, hidden),
        in_norm_w=(rng.uniform(0.5, 1.5, size=hidden) / 128.0).astype(np.float32),
        q_norm_w=rng.uniform(0.5, 1.5, size=D).astype(np.float32),
        k_norm_w=rng.uniform(0.5, 1.5, size=D).astype(np.float32),
        w_out=random_weights(rng, wtype, hidden, Hq * D),
    )


def attn_inputs(rng: np.random.Generator, n_seqs: int, layer: dict, max_ctx: int, pos=None) -> dict:
    """x ~ N(0, 1); fp16 KV caches [n, max_ctx, Hkv, D] pre-filled with
    N(0, 1) keys and values (as uint16 bits); pos[s] (default max_ctx - 1 for
    every sequence) is the slot the step writes."""
    Hkv, D = layer["n_kv_heads"], layer["head_dim"]
    kc = rng.standard_normal((n_seqs, max_ctx, Hkv, D)).astype(np.float16).view(np.uint16)
    vc = rng.standard_normal((n_seqs, max_ctx, Hkv, D)).astype(np.float16).view(np.uint16)
    if pos is None:
        pos = np.full(n_seqs, max_ctx - 1, np.int32)
    return dict(x=rng.standard_normal((n_seqs, layer["hidden"])).astype(np.float32), k_cache=kc, v_cache=vc,
                pos=np.asarray(pos, np.int32))
