"""Shared test setup: puts the repo root on sys.path, registers the `gpu` marker and exposes
the package (directory ``uefi-gpu_b200``) and the CPU oracle (``oracle/pyoracle.py``)."""
from __future__ import annotations

import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (run on the GPU box)")


def load_package():
    return importlib.import_module("uefi-gpu_b200")


def load_oracle():
    from oracle import pyoracle
    return pyoracle


@pytest.fixture(scope="session")
def ugb():
    return load_package()


@pytest.fixture(scope="session")
def orc():
    return load_oracle()


@pytest.fixture(scope="session")
def ctx(ugb):
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    c = ugb.Context(0)
    yield c
    c.close()


def golden(name: str):
    return np.load(os.path.join(GOLDEN, name))


def assert_rows_close(gpu: np.ndarray, ref: np.ndarray, rel: float = 1e-3, terms: np.ndarray | None = None) -> None:
    """Per-row fp32 parity: |gpu - ref| <= rel * max(|ref|, 1e-3 * rms(ref)).

    The contract is 1e-3 relative per row.  Rows whose exact value cancels to below 1e-3 of
    the output's RMS are held to the same absolute error as a row of magnitude 1e-3 * RMS
    (a pure relative bound is meaningless at a zero crossing).  With `terms` (per row, the sum
    of the magnitudes of its block terms, oracle matvec_terms) a cancelling row may also differ
    by rel * 1e-2 * terms: a sum whose blocks are added in another order (split over K) differs
    from the sequential one by about sqrt(blocks) * 2^-24 * terms, 1.4e-6 * terms for 600 blocks."""
    gpu = np.asarray(gpu, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert gpu.shape == ref.shape
    assert np.all(np.isfinite(gpu)), "non-finite GPU output"
    rms = np.sqrt(np.mean(ref * ref)) if ref.size else 0.0
    bound = rel * np.maximum(np.abs(ref), 1e-3 * rms)
    if terms is not None:
        bound = np.maximum(bound, rel * 1e-2 * np.asarray(terms, dtype=np.float64))
    err = np.abs(gpu - ref)
    bad = err > bound
    if np.any(bad):
        i = int(np.argmax(err / np.maximum(bound, 1e-300)))
        raise AssertionError(
            f"{int(bad.sum())} rows outside tolerance; worst index {i}: gpu={gpu.flat[i]!r} "
            f"ref={ref.flat[i]!r} err={err.flat[i]:.3e} bound={bound.flat[i]:.3e}")
