"""Shared test setup.

* registers the `gpu` marker (tests that need a B200) and `slow`;
* puts the operator package (atomic-ops_b200/) and the repository root (for the
  test-only `oracle` package) on sys.path.
"""
import os
import pathlib
import sys

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
PKG_PARENT = ROOT / "atomic-ops_b200"
for p in (str(PKG_PARENT), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device (sm_100a)")
    config.addinivalue_line("markers", "slow: longer CPU test")


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


# Regimes of the reference fixture (tests_gdn2/conftest.py:6-11):
# name, seed, g_scale, k_scale, b_scale, in_domain
SEEDS = [
    ("benign0", 0, 0.05, 1.0, 0.5, True), ("benign1", 1, 0.05, 1.0, 0.5, True),
    ("strong_decay", 2, 3.0, 1.0, 0.5, True), ("near_zero", 3, 0.001, 1.0, 0.5, True),
    ("b_near_one", 5, 0.3, 1.0, 0.95, True), ("large_k_stable", 4, 0.3, 8.0, 0.02, True),
    ("large_kb_OOD", 4, 0.3, 8.0, 4.0, False)]
DOMAIN = [s for s in SEEDS if s[5]]

os.environ.setdefault("PYTHONHASHSEED", "0")
