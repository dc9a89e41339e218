"""The tensor-core depthwise path (csrc/dw_tc.cu, selected by UNOQ_DW_TC=1 at load time; off by
default because the dp4a kernel is faster) against the reference runtime's goldens and the oracle.
Depthwise semantics: runtime/qnn.c:807-983. Bit-exact: integer arithmetic throughout."""
import ctypes as C

import numpy as np
import pytest

import opcases
from conftest import model_path
from gpuhelp import NativeSession

pytestmark = pytest.mark.gpu

# the depthwise cases whose channel count (a multiple of 32) the tensor-core path takes
CASES = ["dw3_s1", "dw5_s1", "dw3_s2_wide", "dw5_s1_post", "dw5_s2_c64", "dw3_s2_c128_img2", "dw3_s1_c256_wide"]


@pytest.fixture
def dw_tc(monkeypatch):
    monkeypatch.setenv("UNOQ_DW_TC", "1")


@pytest.mark.parametrize("name", CASES)
def test_dw_tc_matches_reference_golden(name, dw_tc, native, golden_ops):
    plan = golden_ops[f"{name}/plan"].tobytes()
    x = golden_ops[f"{name}/x"]
    assert native.ug_load(C.create_string_buffer(plan, len(plan)), len(plan)) == 0, native.ug_last_error()
    y = np.empty(native.ug_output_bytes(), dtype=np.int8)
    assert native.ug_run(x.ctypes.data, x.nbytes, y.ctypes.data, y.size) == 0, native.ug_last_error()
    np.testing.assert_array_equal(y, golden_ops[f"{name}/y"])


@pytest.mark.parametrize("name", CASES)
def test_dw_tc_batch_matches_oracle_at_scale(name, dw_tc, native, oracle):
    """Three images at scale 4 (several row tiles per image, and image slots shared by two images
    for the whole-image case) against the oracle."""
    builder = dict(opcases.all_cases(4))[name]
    rng = np.random.default_rng(202)
    plan, x0 = builder(rng)
    xs = np.stack([x0] + [rng.integers(-128, 128, size=x0.shape, dtype=np.int64).astype(np.int8) for _ in range(2)])
    expect = oracle.run(plan, xs, 3)
    with NativeSession(native, plan) as s:
        np.testing.assert_array_equal(s.run(xs, 3), expect)


def test_dw_tc_mobilenetv4_matches_reference(dw_tc, native, golden_models, oracle):
    """MobileNetV4's fifteen depthwise layers through the tensor-core path, whole network: batch 1
    against the reference runtime's outputs, and a batch of 3 against the oracle."""
    from unoq_dsp import load
    model = load(model_path("mobilenetv4-small"))
    rng = np.random.default_rng(0)
    with NativeSession(native, model.plan) as s:
        x0 = np.random.default_rng(0).integers(-128, 128, size=(1, 224, 224, 3), dtype=np.int64).astype(np.int8)
        np.testing.assert_array_equal(s.run(x0), golden_models["mobilenetv4-small/y0"])
        xs = rng.integers(-128, 128, size=(3, 224, 224, 3), dtype=np.int64).astype(np.int8)
        np.testing.assert_array_equal(s.run(xs, 3), oracle.run(model.plan, xs, 3))
