"""Shared fixtures for the gemq-b200 test suite.

Layers (mirroring the reference's ladder, tests/conftest.py:1-12 of RobustGEMQ):
  * oracle vs golden vectors recorded from the reference's own kernels (CPU)
  * C-ABI library loads and exports every declared symbol (CPU)
  * host-side layout / guards / expert-parallel plumbing (CPU, gloo ranks)
  * CUDA kernels vs the oracle, bit-exact dequant, block rel-L2 (``-m gpu``)
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return GOLDEN


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / name) as f:
        return {k: f[k] for k in f.files}


def proj_from(data: dict, prefix: str):
    from oracle import gemq_oracle as O

    return O.PackedProj(
        wq=data[f"{prefix}_wq"], scales=data[f"{prefix}_scales"], zeros=data[f"{prefix}_zeros"],
        nbits=data[f"{prefix}_nbits"], group_sizes=data[f"{prefix}_group_sizes"],
        wq_strides=data[f"{prefix}_wq_strides"], zs_strides=data[f"{prefix}_zs_strides"],
        K=int(data[f"{prefix}_K"]), N=int(data[f"{prefix}_N"]))


def rel_l2(actual, reference) -> float:
    """Frobenius relative error in float64 (the reference's ``relative_error``,
    tests/conftest.py:152-157 of RobustGEMQ)."""
    a = np.asarray(actual, dtype=np.float64)
    r = np.asarray(reference, dtype=np.float64)
    return float(np.linalg.norm(a - r) / max(np.linalg.norm(r), 1e-12))


@pytest.fixture(scope="session")
def cuda_device():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")
