import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("", "oracle", "micro-vllm_b200", os.path.join("tests", "golden")):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)

# Parity tolerance of the north star: <= 1e-2 relative L2 and <= 2e-2 max-abs
# on the f32-accumulated outputs; integer work (routing, permutation) exact.
REL_L2_TOL = 1e-2
MAX_ABS_TOL = 2e-2


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


def max_abs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)))) if np.size(
        a) else 0.0


def assert_close(got, want, what=""):
    r, m = rel_l2(got, want), max_abs(got, want)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    assert r <= REL_L2_TOL and m <= MAX_ABS_TOL, f"{what}: rel_l2={r:.3e} max_abs={m:.3e}"
    return r, m


@pytest.fixture(scope="session")
def port():
    from oracle import Oracle
    return Oracle("port")


@pytest.fixture(scope="session")
def ref():
    from oracle import Oracle, available
    if not available("reference") and not os.path.isdir("/root/reference"):
        pytest.skip("reference build (oracle/_ref) not present")
    return Oracle("reference")


@pytest.fixture(scope="session")
def golden():
    d = os.path.join(ROOT, "tests", "golden")
    arrays = dict(np.load(os.path.join(d, "golden.npz")))
    with open(os.path.join(d, "golden.json")) as f:
        meta = json.load(f)["cases"]
    return arrays, meta


@pytest.fixture(scope="session")
def moe():
    """The CUDA library, initialised on cuda:0 (GPU tests only)."""
    import build as mvbuild
    mvbuild.build()
    import mvllm_moe
    mvllm_moe.init(0)
    return mvllm_moe


@pytest.fixture
def exact(moe):
    """Exact mode for the test (the epilogue and router scores keep the
    reference's order and roundings), the default afterwards."""
    moe.set_exact(True)
    yield moe
    moe.set_exact(None)
