import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
for p in (ROOT, ROOT / "iree-adreno-genai-tuner_b200", GOLDEN):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def load_golden(name):
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def golden_ops():
    return load_golden("q4_ops")


@pytest.fixture(scope="session")
def golden_rope():
    return load_golden("rope")


@pytest.fixture(scope="session")
def golden_gemv():
    return load_golden("gemv_5120x3072")


@pytest.fixture(scope="session", params=["tiny_baseline", "tiny_ref"])
def golden_model(request):
    return request.param, load_golden(f"model_{request.param}")
