"""Shared test set-up: the `gpu` marker, import paths and tolerance helpers."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a); runs through the C ABI")


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def max_rel_err(got, ref) -> float:
    """Normwise relative error max|got - ref| / max|ref| (the tolerance the
    fp32 paths are held to; elementwise relative error is meaningless for
    outputs that cancel to near zero)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    denom = max(np.abs(ref).max(initial=0.0), 1e-30)
    return float(np.abs(got - ref).max(initial=0.0) / denom)


def elementwise_rel_err(got, ref, floor: float = 1e-3) -> float:
    """Largest elementwise relative error |got - ref| / |ref| over the
    elements with |ref| above floor * max|ref| (below that floor an element
    is the residue of cancellation and its relative error says nothing about
    the arithmetic)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    a = np.abs(ref)
    m = a > floor * max(a.max(initial=0.0), 1e-30)
    if not m.any():
        return 0.0
    return float((np.abs(got - ref)[m] / a[m]).max())


def assert_close(got, ref, tol: float, what: str = "") -> None:
    e = max_rel_err(got, ref)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    assert e <= tol, f"{what}: normwise relative error {e:.3e} > {tol:.1e}"


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test run without a CUDA device")
    from leaninfer_b200 import build
    build.build()
    from leaninfer_b200 import _lib
    _lib.load()
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle
    oracle.lib()
    return oracle
