"""The oracle's ggml-style quantized-activation variant (unpinned: no
reference vector fixes ggml's CPU results). Its mechanics are checked
against the exact oracle: activations that its 8-bit grid represents exactly
give the exact dot products; random activations land within the 8-bit
quantization error (and measurably off, so the quantization is active)."""
from __future__ import annotations

import numpy as np
import pytest

from leaninfer_b200 import synth
from oracle import oracle


def _err(a, b):
    return float(np.abs(a - b).max() / np.abs(b).max())


@pytest.mark.parametrize("wtype", [8, 12])
def test_exact_on_representable_activations(wtype):
    r = np.random.Generator(np.random.PCG64(61))
    K, N = 1024, 48
    W = synth.random_weights(r, wtype, N, K)
    qk = 256 if wtype == 12 else 32
    q = r.integers(-126, 127, size=(2, K)).astype(np.float32)
    q[:, ::qk] = -127                      # every block's largest magnitude: -127
    x = q / 128.0                          # step 2^-7: exact in fp32 and in the fp16 block scale
    got = oracle.rms_norm_matmul_q8act(wtype, x, None, W, N)
    ref = oracle.rms_norm_matmul(wtype, x, None, W, N)
    # Q8_0: both are sums of the same exact products; Q4_K: the exact oracle
    # decodes d*sc*q - dmin*m in separately rounded fp32, the variant in integers
    assert _err(got, ref) <= (1e-12 if wtype == 8 else 1e-6)


@pytest.mark.parametrize("wtype", [8, 12])
def test_random_activations_within_8bit_error(wtype):
    r = np.random.Generator(np.random.PCG64(62))
    K, N = 2048, 64
    W = synth.random_weights(r, wtype, N, K)
    x = r.standard_normal((3, K)).astype(np.float32)
    gamma = r.uniform(0.5, 1.5, K).astype(np.float32)
    e = _err(oracle.rms_norm_matmul_q8act(wtype, x, gamma, W, N), oracle.rms_norm_matmul(wtype, x, gamma, W, N))
    assert 1e-4 < e < 3e-2, e
