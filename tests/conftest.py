"""Shared fixtures and markers for the DWA hot-path tests.

``-m gpu`` tests need a CUDA device and the built ``libdwa.so``; everything else
runs on the CPU (oracle against golden vectors, host logic, C-ABI symbols,
``gloo`` multi-process tests).
"""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libdwa.so")


def load_golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN_DIR, f"{name}.npz")) as f:
        return {k: f[k] for k in f.files}


def assert_close(actual, expected, rtol, atol_scale=None, name=""):
    """``|a - e| <= rtol * |e| + atol`` elementwise, with ``atol = rtol *
    atol_scale`` (default: ``rtol * max|e|``), so that entries near zero are
    judged on the tensor's own scale.  Reports the worst element."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    assert a.shape == e.shape, f"{name}: shape {a.shape} != {e.shape}"
    scale = float(np.max(np.abs(e))) if atol_scale is None else float(atol_scale)
    atol = rtol * scale
    err = np.abs(a - e)
    bad = err > rtol * np.abs(e) + atol
    if bad.any():
        i = np.unravel_index(np.argmax(err - rtol * np.abs(e)), err.shape)
        raise AssertionError(
            f"{name}: {int(bad.sum())}/{bad.size} elements out of tolerance (rtol={rtol}, "
            f"atol={atol:.3g}); worst at {i}: got {a[i]!r} expected {e[i]!r}")
