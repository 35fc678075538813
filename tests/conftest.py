"""Shared pytest setup: the ``gpu`` marker, repo-root imports, and the package loader.

GPU tests are marked ``@pytest.mark.gpu``; the CPU suite runs with ``-m "not gpu"``.
"""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_pkg():
    """The package directory is ``llm-gpu-5_b200`` (not an identifier), so import it by name."""
    return importlib.import_module("llm-gpu-5_b200")


@pytest.fixture(scope="session")
def pkg():
    return load_pkg()


@pytest.fixture(scope="session")
def cuda_dev():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
