import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU; run with -m gpu")


def _golden(prefixes):
    names = sorted(f[:-4] for f in os.listdir(GOLDEN) if f.endswith(".npz"))
    return [n for n in names if n.startswith(prefixes)]


@pytest.fixture(scope="session")
def golden_names():
    """The SwiGLU fixtures (tests/golden/make_golden.py)."""
    names = sorted(f[:-4] for f in os.listdir(GOLDEN) if f.endswith(".npz"))
    return [n for n in names if not n.startswith(("rope_", "attention_"))]


@pytest.fixture(scope="session")
def rope_golden_names():
    """The RoPE fixtures (tests/golden/make_golden_rope_attention.py)."""
    return _golden(("rope_",))


@pytest.fixture(scope="session")
def attention_golden_names():
    """The attention fixtures (tests/golden/make_golden_rope_attention.py)."""
    return _golden(("attention_",))


def load_golden(name):
    import numpy as np

    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: z[k] for k in z.files}
