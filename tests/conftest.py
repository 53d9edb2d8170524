"""Shared fixtures. Tests marked ``gpu`` need a B200; everything else runs on
the CPU (oracle vs golden vectors, host logic, C-ABI symbol checks)."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import nvfp4 as O
    O.oracle_lib()
    return O


@pytest.fixture(scope="session")
def sbb():
    import __graft_entry__ as g
    return g.load_package()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test collected on a machine without CUDA")
    return torch.device("cuda", 0)


def golden(name: str) -> dict:
    with np.load(GOLDEN / name) as z:
        return {k: z[k] for k in z.files}


def rel_err(got: np.ndarray, want: np.ndarray) -> float:
    """max |got - want| / max |want| (the normwise max relative error)."""
    return float(np.abs(got.astype(np.float64) - want).max() / max(np.abs(want).max(), 1e-30))


def cosine(got: np.ndarray, want: np.ndarray) -> float:
    a = got.astype(np.float64).ravel()
    b = want.astype(np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))
