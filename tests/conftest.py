import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")


def _gpu_available() -> bool:
    try:
        import torch

        return bool(torch.cuda.is_available())
    except Exception:  # pragma: no cover
        return False


def pytest_collection_modifyitems(config, items):
    if _gpu_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    cache = {}

    def load(name):
        if name not in cache:
            cache[name] = dict(np.load(GOLDEN / name, allow_pickle=False))
        return cache[name]

    return load


@pytest.fixture(scope="session")
def oracle_c():
    """ctypes handle on the plain-C oracle (built by ``make -C oracle``)."""
    import ctypes
    import subprocess

    lib = REPO / "oracle" / "libmaxsim_oracle.so"
    if not lib.exists():
        subprocess.run(["make", "-C", str(REPO / "oracle"), "libmaxsim_oracle.so"], check=True,
                       stdout=subprocess.DEVNULL)
    return ctypes.CDLL(str(lib))
