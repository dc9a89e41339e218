import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "unoq-dsp_b200", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = ROOT / "tests" / "golden"
MODELS = ROOT / "models"
LIB = ROOT / "unoq-dsp_b200" / "lib" / "libunoq_cuda.so"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def golden_ops():
    return np.load(GOLDEN / "ops.npz")


@pytest.fixture(scope="session")
def golden_models():
    return np.load(GOLDEN / "models.npz")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle, ORACLE_LIB
    if not ORACLE_LIB.is_file():
        pytest.fail("oracle/liboracle.so missing: run `make -C oracle` (or __graft_entry__.build())")
    return Oracle()


@pytest.fixture(scope="session")
def native():
    from unoq_dsp.native import load_library
    if not LIB.is_file():
        pytest.fail("libunoq_cuda.so missing: run unoq-dsp_b200/build.py (or __graft_entry__.build())")
    return load_library(LIB)


def model_path(name):
    p = MODELS / f"{name}.uqmodel"
    if not p.is_file():
        pytest.skip(f"{p} not staged (build() copies the bundled models when the reference is mounted)")
    return p
