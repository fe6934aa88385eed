"""Test configuration: registers the `gpu` marker and puts the host package and
the oracle on sys.path. The product library is built in place if missing
(nvcc cross-compiles without a GPU); GPU tests then load it and fail loudly if
anything is absent -- there is no fallback path."""
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "cuda-operators_b200"
sys.path.insert(0, str(PKG))
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (sm_100a)")
    if not (PKG / "libkvdecode_b200.so").exists():
        subprocess.run(["make", "-C", str(PKG), "-j8"], check=True)
    if not (ROOT / "oracle" / "libkvd_oracle.so").exists():
        subprocess.run(["make", "-C", str(ROOT / "oracle"), "oracle"], check=True)


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return dict(np.load(ROOT / "tests" / "golden" / "kv_golden.npz"))
