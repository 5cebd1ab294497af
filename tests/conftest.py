"""Shared test setup: import paths, the `gpu` marker, build-on-demand of the CUDA library
and of the CPU oracle (the oracle is test infrastructure: tests use it only as the checker)."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "ane-training-experiments_b200"
for p in (str(PKG), str(REPO / "oracle"), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def _ensure_built():
    lib = PKG / "lib" / "libllm_cuda.so"
    if not lib.exists():
        subprocess.run(["make", "-s", "-C", str(PKG)], check=True)
    orc = REPO / "oracle" / "_build" / "liboracle.so"
    if not orc.exists():
        subprocess.run(["make", "-s", "-C", str(REPO / "oracle")], check=True)


_ensure_built()


@pytest.fixture(scope="session")
def gpu_available():
    import torch
    return torch.cuda.is_available()
