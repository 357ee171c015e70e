"""Shared fixtures.  Tests marked `gpu` need a CUDA device (B200); the rest run
on the CPU.  The reference's own suite seeds torch with 42 for every test
(tests/conftest.py:16-21 of mach9robotics/msda-triton); so does this one."""

from __future__ import annotations

import glob
import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs on the B200 box)")
    config.addinivalue_line("markers", "slow: long-running")


@pytest.fixture(autouse=True)
def seed_rng() -> None:
    torch.manual_seed(42)
    if torch.cuda.is_available():
        torch.cuda.manual_seed(42)


@pytest.fixture
def cuda_device():
    if not torch.cuda.is_available():
        pytest.fail("test marked gpu but CUDA is not available")
    return torch.device("cuda", 0)


def golden_names() -> list[str]:
    return sorted(os.path.basename(f)[:-4] for f in glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


def load_golden(name: str) -> dict:
    z = np.load(os.path.join(GOLDEN_DIR, f"{name}.npz"))
    return {k: z[k] for k in z.files}
