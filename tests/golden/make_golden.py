"""Generates the committed golden fixtures under tests/golden/.

Run in a container that has the third-party pins installed and the reference
checkout mounted (the GPU box has neither, so the outputs are committed):

    python tests/golden/make_golden.py

Pins, one fixture each:
  dequant_q8_0.npz / dequant_q4_k.npz
      gguf-py 0.19.0 (gguf/quants.py: Q8_0.dequantize_blocks :396,
      Q4_K.get_scale_min :479 and dequantize_blocks :503) on random blocks plus
      edge blocks (zero, subnormal, negative and extreme scales; every code).
  gdr_recurrent.npz
      flash-linear-attention 0.5.1 naive_recurrent_gated_delta_rule
      (fla/ops/gated_delta_rule/naive.py:13), inputs mapped to the reference
      kernel's layouts (cuda/leaninfer-fused-deltanet.cu:170-189): beta given
      as a logit (the reference applies the sigmoid, :235), g as log-decay.
  gdr_chunk.npz
      the same library's naive_chunk_gated_delta_rule (naive.py:67, chunk 64,
      T not a multiple of the chunk) - the WY chunk form the prefill follows.
  ref_cpu_swiglu.npz
      the reference's own CPU function cpu_rms_norm_swiglu
      (cuda/benchmark_fused.cu:99-121), compiled from the reference sources by
      oracle/Makefile (`make -C oracle ref`).
All inputs come from numpy.random.Generator(PCG64(seed)).
"""
from __future__ import annotations

import sys
import warnings
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def fp16_bytes(v) -> np.ndarray:
    return np.asarray(v, dtype=np.float16).view(np.uint8).reshape(-1, 2)


def q8_0_blocks(r: np.random.Generator) -> np.ndarray:
    n_rand = 256
    d = r.uniform(-2e-2, 2e-2, n_rand).astype(np.float16)
    qs = r.integers(0, 256, (n_rand, 32), dtype=np.int16).astype(np.uint8)
    blocks = [np.concatenate([fp16_bytes(d), qs], axis=1)]
    # edge blocks: every int8 code (8 blocks x 32 = 256 codes) under assorted scales
    edge_d = np.array([1.0, -1.0, 0.0, 6.1e-05, 5.96e-08, -3.0e-06, 65504.0, 1e-3], np.float16)
    codes = np.arange(256, dtype=np.uint16).astype(np.uint8).reshape(8, 32)
    blocks.append(np.concatenate([fp16_bytes(edge_d), codes], axis=1))
    return np.ascontiguousarray(np.concatenate(blocks, axis=0))


def q4_k_blocks(r: np.random.Generator) -> np.ndarray:
    n_rand = 128
    d = r.uniform(-2e-2, 2e-2, n_rand).astype(np.float16)
    dmin = r.uniform(-2e-2, 2e-2, n_rand).astype(np.float16)
    sc = r.integers(0, 256, (n_rand, 12), dtype=np.int16).astype(np.uint8)
    qs = r.integers(0, 256, (n_rand, 128), dtype=np.int16).astype(np.uint8)
    blocks = [np.concatenate([fp16_bytes(d), fp16_bytes(dmin), sc, qs], axis=1)]
    # edge blocks: all-ones / all-zero scale bytes, every nibble, tiny and huge d
    e_d = np.array([1.0, 0.0, 6.1e-05, 5.96e-08, 1000.0, -0.5], np.float16)
    e_m = np.array([0.5, 1.0, -6.1e-05, 0.0, 65504.0, 0.25], np.float16)
    e_sc = np.stack([np.full(12, 0xFF, np.uint8), np.zeros(12, np.uint8),
                     np.arange(12, dtype=np.uint8) * 21, np.full(12, 0xC0, np.uint8),
                     np.full(12, 0x3F, np.uint8), np.arange(12, dtype=np.uint8)[::-1] * 17])
    e_qs = np.stack([np.arange(128, dtype=np.uint8) * 2 + (i % 2) for i in range(6)]).astype(np.uint8)
    blocks.append(np.concatenate([fp16_bytes(e_d), fp16_bytes(e_m), e_sc, e_qs], axis=1))
    return np.ascontiguousarray(np.concatenate(blocks, axis=0))


def make_dequant() -> None:
    from gguf.constants import GGMLQuantizationType
    from gguf.quants import dequantize

    b8 = q8_0_blocks(rng(11))
    ref8 = dequantize(b8.reshape(-1), GGMLQuantizationType.Q8_0).astype(np.float32)
    np.savez_compressed(HERE / "dequant_q8_0.npz", blocks=b8, values=ref8.reshape(-1))
    b4 = q4_k_blocks(rng(12))
    ref4 = dequantize(b4.reshape(-1), GGMLQuantizationType.Q4_K).astype(np.float32)
    np.savez_compressed(HERE / "dequant_q4_k.npz", blocks=b4, values=ref4.reshape(-1))


def make_recurrent() -> None:
    import torch
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        from fla.ops.gated_delta_rule.naive import naive_recurrent_gated_delta_rule

    cases = {}
    for name, (B, T, H, D) in {"d128": (1, 4, 2, 128), "d64": (2, 5, 2, 64)}.items():
        r = rng(21 + D)
        q = r.standard_normal((B, T, H, D)).astype(np.float32)
        k = r.standard_normal((B, T, H, D)).astype(np.float32)
        k /= np.linalg.norm(k, axis=-1, keepdims=True)
        q /= np.linalg.norm(q, axis=-1, keepdims=True)
        v = r.standard_normal((B, T, H, D)).astype(np.float32)
        beta_logit = r.standard_normal((B, T, H)).astype(np.float32)
        g = (-np.log1p(np.exp(r.standard_normal((B, T, H)))) *
             np.exp(r.normal(0, 0.5, (B, T, H)))).astype(np.float32)
        s0 = r.normal(0, 0.02, (B, H, D, D)).astype(np.float32)
        beta = 1.0 / (1.0 + np.exp(-beta_logit.astype(np.float64)))
        o, sT = naive_recurrent_gated_delta_rule(
            torch.from_numpy(q).double(), torch.from_numpy(k).double(), torch.from_numpy(v).double(),
            torch.from_numpy(beta).double(), torch.from_numpy(g).double(), scale=D ** -0.5,
            initial_state=torch.from_numpy(s0).double(), output_final_state=True)
        # reference layouts: q,k [B][H][T][D]; v same with element strides;
        # g,beta [B][T][H]; state [B][H][D][D]; out [B][T][H][D]
        cases[name] = dict(
            q=np.ascontiguousarray(q.transpose(0, 2, 1, 3)), k=np.ascontiguousarray(k.transpose(0, 2, 1, 3)),
            v=np.ascontiguousarray(v.transpose(0, 2, 1, 3)), g=g, beta_logit=beta_logit, state=s0,
            out=o.float().numpy(), state_out=sT.float().numpy(), dims=np.array([B, T, H, D]))
    np.savez_compressed(HERE / "gdr_recurrent.npz",
                        **{f"{c}_{k}": v for c, d in cases.items() for k, v in d.items()})


def make_chunk() -> None:
    import torch
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        from fla.ops.gated_delta_rule.naive import naive_chunk_gated_delta_rule

    T, H, D = 130, 2, 64
    r = rng(31)
    bf = lambda a: torch.from_numpy(a).to(torch.bfloat16)
    q = r.standard_normal((1, T, H, D)).astype(np.float32)
    k = r.standard_normal((1, T, H, D)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = r.standard_normal((1, T, H, D)).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-r.standard_normal((1, T, H))))).astype(np.float32)
    g = (-np.log1p(np.exp(r.standard_normal((1, T, H)))) * np.exp(r.normal(0, 0.5, (1, T, H)))).astype(np.float32)
    s0 = r.normal(0, 0.02, (1, H, D, D)).astype(np.float32)
    qb, kb, vb = bf(q), bf(k), bf(v)
    o, sT = naive_chunk_gated_delta_rule(qb.double(), kb.double(), vb.double(), torch.from_numpy(g).double(),
                                         torch.from_numpy(beta).double(), chunk_size=64, scale=D ** -0.5,
                                         initial_state=torch.from_numpy(s0).double(), output_final_state=True)
    np.savez_compressed(HERE / "gdr_chunk.npz",
                        q=qb.view(torch.int16).numpy().view(np.uint16)[0],
                        k=kb.view(torch.int16).numpy().view(np.uint16)[0],
                        v=vb.view(torch.int16).numpy().view(np.uint16)[0],
                        g=g[0], beta=beta[0], state=s0[0], out=o.float().numpy()[0],
                        state_out=sT.float().numpy()[0])


def make_ref_cpu() -> None:
    from oracle import oracle

    if not oracle.REF_BENCH.exists():
        oracle.build(with_ref=True)
    r = rng(41)
    K, N, eps = 256, 64, 1e-5
    x = ((r.random(K) - 0.5) * 0.1).astype(np.float32)
    gamma = (1.0 + (r.random(K) - 0.5) * 0.01).astype(np.float32)
    Wg = ((r.random((N, K)) - 0.5) * 0.02).astype(np.float32)
    Wu = ((r.random((N, K)) - 0.5) * 0.02).astype(np.float32)
    out = oracle.ref_cpu_rms_norm_swiglu(x, gamma, Wg, Wu, eps)
    np.savez_compressed(HERE / "ref_cpu_swiglu.npz", x=x, gamma=gamma, Wg=Wg, Wu=Wu, eps=np.float32(eps), out=out)


if __name__ == "__main__":
    make_dequant()
    make_recurrent()
    make_chunk()
    make_ref_cpu()
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)
