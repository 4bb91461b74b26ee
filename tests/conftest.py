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


def assert_close_bf16_out(got, want, max_abs=MAX_ABS, rel_l2=REL_L2, what=""):
    """assert_close for an output the path rounds to bf16 (the residual stream
    of the decode stacks, |y| up to ~10): the max-abs bar plus one bf16 ulp of
    the oracle value (2^-7 |want|), the rounding of an f32 result to bf16; the
    relative-L2 bar unchanged."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    err = np.abs(got - want)
    bound = max_abs + np.abs(want) * 2.0 ** -7
    worst = float((err - bound).max(initial=-1.0))
    _, rl = close_report(got, want)
    assert worst <= 0 and rl <= rel_l2, (f"{what}: max excess over the bound {worst:.3e}, "
                                         f"max_abs={err.max(initial=0.0):.3e} rel_l2={rl:.3e}")


def check_routing(orc, x_bits, G_bits, bias, inds, wts, k):
    """GPU routing [T, k] against the oracle router (Laguna.swift:165-180) on the
    same x (bf16 bits [T, H]).  The GPU sums the logits in another order than
    the oracle, so a logit may round to the neighbouring bf16 value: an expert
    may differ from the oracle's set only where its choice lies within one
    such rounding step (sigmoid' <= 1/4 times the bf16 spacing of the logit,
    2^-7 |logit|) of the k-th choice, and the weights of an equal set agree
    to that step.  Returns (oracle inds, oracle weights)."""
    b = np.asarray(bias, np.float32)
    oi, ow, logits = orc.port.router_topk(x_bits, G_bits, b, k)
    gi = np.asarray(inds).reshape(oi.shape)
    gw = np.asarray(wts).reshape(ow.shape)
    s = 1.0 / (1.0 + np.exp(-logits.astype(np.float64)))
    choice = s + b
    step = 0.25 * 2.0 ** -7 * np.maximum(np.abs(logits), 1e-3)
    for t in range(oi.shape[0]):
        kth = np.sort(choice[t])[::-1][k - 1]
        diff = set(gi[t].tolist()) ^ set(oi[t].tolist())
        for e in diff:
            assert abs(choice[t, e] - kth) <= step[t, e] + 1e-6, (t, e, choice[t, e], kth)
        if not diff:
            order = {e: j for j, e in enumerate(oi[t])}
            np.testing.assert_allclose(gw[t], ow[t][[order[e] for e in gi[t]]], rtol=1e-2,
                                       atol=1e-6)
    return oi, ow
