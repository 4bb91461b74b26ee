import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "nvfp4_golden.npz")
PKG = "mlxfast-challenge_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def _build_once():
    import subprocess
    mk = os.path.join(ROOT, "oracle", "Makefile")
    if not os.path.exists(os.path.join(ROOT, "oracle", "liboracle.so")):
        subprocess.run(["make", "-s", "-f", mk, os.path.join(ROOT, "oracle", "liboracle.so")],
                       check=True)
    build = importlib.import_module(PKG + ".build")
    build.build()


@pytest.fixture(scope="session")
def nv():
    _build_once()
    return importlib.import_module(PKG)


@pytest.fixture(scope="session")
def orc():
    _build_once()
    import oracle
    importlib.reload(oracle)
    assert oracle.port is not None, "oracle/liboracle.so failed to load"
    return oracle


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN))


def close_report(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want)
    rel_l2 = np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)
    return float(err.max(initial=0.0)), float(rel_l2)


# Output tolerance stated for this path: max-abs <= 2e-2 and relative-L2 <= 5e-3
# against the fp32-accumulated oracle.
MAX_ABS = 2e-2
REL_L2 = 5e-3


def assert_close(got, want, max_abs=MAX_ABS, rel_l2=REL_L2, what=""):
    ma, rl = close_report(got, want)
    assert ma <= max_abs and rl <= rel_l2, f"{what}: max_abs={ma:.3e} rel_l2={rl:.3e}"
