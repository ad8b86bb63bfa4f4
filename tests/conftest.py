"""Shared test setup.

Markers: `gpu` tests run on a B200 and call libkai_gdn_cuda.so through its C
ABI; everything else runs on CPU (the oracle, the host logic, the ABI surface).
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built library")


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    nb = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (nb if nb > 0 else 1.0))


def kai_close(got, ref, abs_tol, rel_tol) -> bool:
    """approx_eq of kleidiai_submission/test_kai_gdn.c:57-62, elementwise."""
    got = np.asarray(got, np.float32)
    ref = np.asarray(ref, np.float32)
    diff = np.abs(got - ref)
    mag = np.maximum(np.abs(got), np.abs(ref))
    return bool(np.all((diff <= abs_tol) | (diff <= rel_tol * mag)))


def validate_pass(got, ref, atol=1e-4, rtol=1e-3) -> bool:
    """compute_error pass rule of gpu/gdn_gpu_validate.c:128-146: fail only if
    max_abs > atol AND max_rel (over |ref| > 1e-2) > rtol."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    d = np.abs(got - ref)
    max_abs = d.max() if d.size else 0.0
    big = np.abs(ref) > 1e-2
    max_rel = (d[big] / np.abs(ref[big])).max() if big.any() else 0.0
    return not (max_abs > atol and max_rel > rtol)


@pytest.fixture(scope="session")
def orc():
    import oracle
    o, _ = oracle.require()
    return o


@pytest.fixture(scope="session")
def ref():
    import oracle
    oracle.require()
    return oracle.ref


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return dict(np.load(GOLDEN / name))
    return load


@pytest.fixture(scope="session")
def lib():
    from orionsbelt_b200 import _lib
    return _lib.lib()


@pytest.fixture(scope="session")
def cuda():
    import torch
    assert torch.cuda.is_available(), "gpu test without a CUDA device"
    torch.cuda.init()
    return torch
