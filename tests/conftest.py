"""Shared pytest configuration.

Tests marked ``gpu`` need a CUDA device (a B200 for the performance-relevant
paths); they are skipped when none is visible. Everything else runs on CPU.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def reference_checkout() -> Path | None:
    """The reference's source tree (``src/qrbench`` + ``scripts/``), if present:
    ``$QRBENCH_REFERENCE``, else the git-ignored ``baseline/_ref/gpumode_qr``
    copy that travels with the repository to GPU boxes. None when neither has
    ``scripts/run_baseline.py``."""
    cands = []
    if os.environ.get("QRBENCH_REFERENCE"):
        cands.append(Path(os.environ["QRBENCH_REFERENCE"]))
    cands.append(REPO / "baseline" / "_ref" / "gpumode_qr")
    for c in cands:
        if (c / "scripts" / "run_baseline.py").exists() and (c / "src" / "qrbench").exists():
            return c.resolve()
    return None


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); skipped without one")
    config.addinivalue_line("markers", "slow: long-running case")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # noqa: BLE001
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device visible")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def load_golden(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / name) as f:
        return {k: f[k] for k in f.files}


def golden_cases(data: dict[str, np.ndarray]) -> list[str]:
    return sorted({k.rsplit("_", 1)[0] for k in data})


@pytest.fixture(scope="session")
def ref_fused():
    return load_golden("ref_fused.npz")


@pytest.fixture(scope="session")
def ref_panel():
    return load_golden("ref_panel.npz")


@pytest.fixture(scope="session")
def ref_blocked():
    return load_golden("ref_blocked.npz")


@pytest.fixture(scope="session")
def lapack_golden():
    return load_golden("lapack.npz")
