import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (run with -m gpu)")


@pytest.fixture(scope="session")
def oracle():
    from oracle import binding
    return binding


@pytest.fixture(scope="session")
def golden_kat():
    import json
    return json.loads((GOLDEN / "ops_kat.json").read_text())


@pytest.fixture(scope="session")
def golden_random():
    return dict(np.load(GOLDEN / "ops_random.npz"))


@pytest.fixture(scope="session")
def golden_tiny():
    return dict(np.load(GOLDEN / "tiny_decode.npz"))


@pytest.fixture(scope="session")
def golden_rotation():
    return dict(np.load(GOLDEN / "rotation_decode.npz"))


@pytest.fixture(scope="session")
def gpu():
    import laplacesscissors_b200 as lsx
    g = lsx.Gpu(0)
    yield g


def close(actual, expected, tolerance):
    """tests/gpu.rs:9-18: |a - e| <= tol * (1 + |e|) elementwise, all finite."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    assert a.shape == e.shape, (a.shape, e.shape)
    assert np.all(np.isfinite(a))
    bad = np.abs(a - e) > tolerance * (1 + np.abs(e))
    assert not bad.any(), f"{int(bad.sum())} elements off; first {np.argmax(bad)}: {a[bad][:4]} vs {e[bad][:4]}"
