"""Shared test configuration.

Markers: ``gpu`` -- needs an sm_100 GPU (the driver runs ``-m gpu`` on a B200
and ``-m "not gpu"`` on a CPU-only box).  The product package lives in a
directory whose name has hyphens, so it is imported with importlib.
"""
from __future__ import annotations

import importlib
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "reference_vectors.npz"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: requires an NVIDIA B200 (sm_100a) GPU")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="CUDA required")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_kl():
    return importlib.import_module("gpu-kernel-lab_b200")


@pytest.fixture(scope="session")
def kl():
    return load_kl()


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)


def bf16_ulp(v: np.ndarray) -> np.ndarray:
    """One bf16 unit in the last place at magnitude |v| (8 significant bits)."""
    a = np.maximum(np.abs(v).astype(np.float64), 2.0 ** -126)
    return 2.0 ** (np.floor(np.log2(a)) - 7)


def assert_matches_oracle(actual, ref_f32, atol=2e-2, rel_frob=5e-3, what=""):
    """The BASELINE gate: max-abs error <= atol (one bf16 ulp where the output
    magnitude makes a single rounding step larger than atol) and relative
    Frobenius error <= rel_frob, against the fp32-accumulated reference."""
    a = actual.float().cpu().numpy() if isinstance(actual, torch.Tensor) else np.asarray(actual, np.float32)
    r = np.asarray(ref_f32, np.float32)
    assert a.shape == r.shape, (a.shape, r.shape)
    err = np.abs(a.astype(np.float64) - r)
    allowed = np.maximum(atol, bf16_ulp(r))
    bad = err > allowed
    if bad.any():
        i = np.unravel_index(np.argmax(err - allowed), err.shape)
        raise AssertionError(f"{what}: {int(bad.sum())} elements over tolerance; worst at {i}: "
                             f"got {a[i]}, ref {r[i]}, err {err[i]:.4g}, allowed {allowed[i]:.4g}")
    denom = max(np.linalg.norm(r.astype(np.float64)), 1e-30)
    rel = np.linalg.norm(a.astype(np.float64) - r) / denom
    assert rel <= rel_frob, f"{what}: rel-Frobenius {rel:.3g} > {rel_frob}"
    return float(err.max()), float(rel)
