import functools
import os
import shutil
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "bnn-train-infer_b200"
for p in (str(PKG), str(ROOT / "oracle"), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (run on the GPU box)")


@functools.lru_cache(maxsize=1)
def gpu_present():
    if shutil.which("nvidia-smi") is None:
        return False
    try:
        out = subprocess.run(["nvidia-smi", "-L"], capture_output=True, text=True, timeout=30)
    except Exception:
        return False
    return out.returncode == 0 and "GPU" in out.stdout


def pytest_collection_modifyitems(config, items):
    if gpu_present():
        return
    skip = pytest.mark.skip(reason="no CUDA device on this host")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle
    return oracle


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return dict(np.load(ROOT / "tests" / "golden" / "rtl_case.npz"))


@pytest.fixture(scope="session")
def b200_device():
    from bnn_b200 import accel
    dev = accel.Device(int(os.environ.get("BNN_TEST_DEVICE", "0")))
    yield dev
    dev.close()
