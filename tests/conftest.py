"""pytest configuration: the `gpu` marker and shared helpers.

`-m "not gpu"` runs everything that needs no GPU (oracle against golden
vectors, host logic, C-ABI loading); `-m gpu` runs the parity tests through
the C ABI on a B200.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA GPU in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def dev():
    import torch

    return torch.device("cuda:0")


def to_dev(a: np.ndarray, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def tol_check(y: np.ndarray, y64: np.ndarray, scale: np.ndarray, rel: float = 1e-5):
    """|y - y64| <= rel * sum|w||x| per row (the row's |w|.|x| scale)."""
    err = np.abs(y.astype(np.float64) - y64) / np.maximum(scale, 1e-30)
    assert np.isfinite(y).all(), "non-finite outputs"
    assert err.max() <= rel, f"max error {err.max():.3e} of |w|.|x| scale exceeds {rel:g}"
    return float(err.max())
