"""Shared pytest setup: import paths, the `gpu` marker, tolerance helpers."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "voxcpm2-c_b200"), os.path.join(REPO, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


def assert_matmul_close(y, y_ref, absscale, tol, what=""):
    """North-star rule: |y - y_ref| <= tol * max(|y_ref|, sum_k |w x| / sqrt(K)), per element."""
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    bound = tol * np.maximum(np.abs(y_ref), np.asarray(absscale, dtype=np.float64))
    err = np.abs(y - y_ref)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err / np.maximum(bound, 1e-300)), err.shape)
        raise AssertionError(f"{what}: {int(bad.sum())} of {bad.size} elements beyond tol {tol}; worst at {i}: "
                             f"y={y[i]!r} ref={y_ref[i]!r} bound={bound[i]!r}")
    return float((err / np.maximum(bound / tol, 1e-300)).max())
