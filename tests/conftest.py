"""Shared pytest setup: the gpu marker, import paths and seeded input helpers."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "ipu-stack_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def seeded_normal(seed, shape, std=1.0):
    return (np.random.default_rng(seed).standard_normal(shape) * std).astype(np.float32)


def seeded_uniform(seed, shape, lo=-1.0, hi=1.0):
    return np.random.default_rng(seed).uniform(lo, hi, shape).astype(np.float32)


def f16_close(actual, ref, max_rel=2e-2, rel_l2=5e-3):
    """BASELINE FP16 tolerance: max|err| <= 2e-2 * max|ref| and rel-L2 <= 5e-3."""
    actual = np.asarray(actual, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(actual - ref)
    scale = max(np.abs(ref).max(), 1e-30)
    l2 = np.linalg.norm(actual - ref) / max(np.linalg.norm(ref), 1e-30)
    ok = err.max() <= max_rel * scale and l2 <= rel_l2
    return ok, f"max|err|={err.max():.4g} (limit {max_rel * scale:.4g}) relL2={l2:.4g} (limit {rel_l2})"
