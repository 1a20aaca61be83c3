"""Shared pytest configuration.

Markers:
  gpu  — needs a CUDA device (B200); run with ``-m gpu``. Everything else runs on CPU.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: test needs a CUDA GPU (sm_100a)")


def rel_l2(ref, got) -> float:
    """||ref - got|| / ||ref|| in float64 (the reference's compute_relative_error,
    nvsubquadratic/testing/utils.py:21-54, evaluated in higher precision)."""
    import torch

    r = ref.detach().double().cpu()
    g = got.detach().double().cpu()
    dn = torch.linalg.norm(r - g).item()
    rn = torch.linalg.norm(r).item()
    return dn if rn < 1e-10 else dn / rn


@pytest.fixture(scope="session")
def golden():
    import torch

    here = os.path.join(ROOT, "tests", "golden")
    return {
        name: torch.load(os.path.join(here, f"{name}.pt"), weights_only=False)
        for name in ("ops", "hyena", "cp", "boundary", "siren")
    }
