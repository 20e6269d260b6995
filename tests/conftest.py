"""pytest configuration.

Markers:
  gpu — needs a CUDA device (the B200 parity tests; run with `-m gpu`).
Everything unmarked runs on a CPU-only machine: the oracle against the golden
vectors, host-side validation of the drop-in API, the C-ABI symbol table and
the multi-rank sharding logic on gloo.
"""

from __future__ import annotations

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(REPO, "simd-ml-kernels_b200")
for p in (REPO, PKG_ROOT, os.path.join(REPO, "oracle"), os.path.join(REPO, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def pytest_report_header(config):
    try:
        import simd_ml_kernels as sk
        return f"simd_ml_kernels (B200): {sk.__file__}"
    except Exception as exc:  # noqa: BLE001
        return f"simd_ml_kernels (B200): not importable ({exc})"


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
