"""Shared fixtures: the CPU oracle, the reference build, golden fixtures, tolerances.

Parity bar (north star: "max relative error 1e-4, fp32 accumulation-order
tolerance"): a device linear output y passes against the reference output r
when BOTH
    max_i |y_i - r_i| / max_i |r_i|              <= 1e-4
    |y_i - r_i| <= 1e-4 * sum_k |w_ik x_k| + 1e-6   for every i
(the second bound is condition-aware: plain per-element relative error is
ill-posed where r_i is near 0). Integer and byte outputs (packing, layout
round trips) must be bit-identical.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"
REL_TOL = 1e-4
ABS_FLOOR = 1e-6


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs through the CUDA library)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle, build

    build()  # no-op when up to date; also builds the reference checker where its sources exist
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle import Reference, reference_available

    if not reference_available():
        pytest.skip("reference build (oracle/_ref) not present")
    return Reference()


@pytest.fixture(scope="session")
def golden():
    from oracle import NAMES, QTYPES

    return {q: dict(np.load(GOLDEN / f"golden_{NAMES[q]}.npz")) for q in QTYPES}


@pytest.fixture(scope="session")
def mq():
    """The product library (built in-tree if stale)."""
    from mini_ai_b200 import build as _build

    _build.build()
    import mini_ai_b200

    mini_ai_b200.lib()
    return mini_ai_b200


def case_names(d: dict) -> list[str]:
    return sorted({k.split("/")[0] for k in d if k.endswith("/y")})


def abs_dot_bound(dequant: np.ndarray, x: np.ndarray) -> np.ndarray:
    """sum_k |w_nk x_mk| for every (m, n), in float64."""
    return np.abs(np.atleast_2d(x).astype(np.float64)) @ np.abs(dequant.astype(np.float64)).T


def assert_linear_close(y: np.ndarray, ref: np.ndarray, bound: np.ndarray, rel: float = REL_TOL) -> dict:
    y = np.asarray(y, dtype=np.float64).reshape(ref.shape)
    ref = np.asarray(ref, dtype=np.float64)
    assert np.all(np.isfinite(y)), "non-finite output"
    err = np.abs(y - ref)
    scale = max(float(np.max(np.abs(ref))), 1e-30)
    max_rel = float(np.max(err)) / scale
    worst = float(np.max(err / (rel * bound + ABS_FLOOR)))
    assert max_rel <= rel, f"max|dy|/max|y| = {max_rel:.3e} > {rel:g}"
    assert worst <= 1.0, f"per-element bound exceeded by {worst:.3f}x (max|dy| = {float(np.max(err)):.3e})"
    return {"max_rel": max_rel, "bound_frac": worst}


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    assert torch.cuda.is_available(), "GPU test needs CUDA"
    return int(os.environ.get("MQ_TEST_DEVICE", "0"))
