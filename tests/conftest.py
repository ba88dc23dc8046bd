"""Shared test setup.

* registers the ``gpu`` marker (tests that need a B200);
* puts the package directory and ``oracle/`` on ``sys.path``;
* builds ``oracle/libgdn_oracle.so`` (gcc) and the package's ``libgdn_b200.so``
  (nvcc, sm_100a) when they are missing, so a fresh checkout can run the CPU
  suite directly.
"""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "qwen38-gdn-dual-sequence-output-tail_b200")
ORACLE = os.path.join(ROOT, "oracle")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (PKG, ORACLE):
    if p not in sys.path:
        sys.path.insert(0, p)


def _ensure_built():
    if not os.path.exists(os.path.join(ORACLE, "libgdn_oracle.so")):
        subprocess.run(["make", "-s", "-C", ORACLE], check=True)
    if not os.path.exists(os.path.join(PKG, "libgdn_b200.so")):
        subprocess.run(["make", "-s", "-C", PKG], check=True)


_ensure_built()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a)")


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but CUDA is not available")
    return torch.device("cuda:0")
