"""ug_run_static, the allocation-free variant of ug_run (fixed 16 MiB device arena, direct
launches), against ug_run on the same graph: identical bytes on two calls in a row, with
ug_run interleaved, for op plans and both bundled models. Collected last on purpose: it must pass
alone and after every other test of the session."""
import ctypes as C

import numpy as np
import pytest

from conftest import model_path

pytestmark = pytest.mark.gpu
OPS = ["block", "conv_stem_rgb", "conv_3x3_s2", "dw5_s1", "add", "concat_c", "transpose_nchw", "softmax_exact",
       "bmm", "pack"]


def _load(native, plan):
    buf = C.create_string_buffer(plan, len(plan))
    assert native.ug_load(buf, len(plan)) == 0, native.ug_last_error()
    return buf


def _run(native, fn, x):
    y = np.empty(native.ug_output_bytes(), dtype=np.int8)
    x = np.ascontiguousarray(x).reshape(-1).view(np.int8)
    rc = fn(x.ctypes.data, x.nbytes, y.ctypes.data, y.nbytes)
    assert rc == 0, (rc, native.ug_last_error())
    return y


@pytest.mark.parametrize("name", OPS)
def test_static_run_equals_ug_run(name, native, golden_ops):
    plan, x = golden_ops[f"{name}/plan"].tobytes(), golden_ops[f"{name}/x"]
    x2 = np.random.default_rng(5).integers(-128, 128, size=x.size, dtype=np.int64).astype(np.int8)
    keep = _load(native, plan)  # noqa: F841  (plan bytes stay alive while loaded)
    first = _run(native, native.ug_run_static, x)
    second = _run(native, native.ug_run_static, x2)
    np.testing.assert_array_equal(first, golden_ops[f"{name}/y"])
    np.testing.assert_array_equal(first, _run(native, native.ug_run, x))
    np.testing.assert_array_equal(second, _run(native, native.ug_run, x2))
    np.testing.assert_array_equal(first, _run(native, native.ug_run_static, x))  # after ug_run


@pytest.mark.parametrize("name,shape", [("mobilenetv4-small", (1, 224, 224, 3)), ("yolo26n-320", (1, 320, 320, 3))])
def test_static_run_on_bundled_models(name, shape, native, golden_models):
    from unoq_dsp import load
    plan = load(model_path(name)).plan
    keep = _load(native, plan)  # noqa: F841
    for seed in (0, 1):
        x = np.random.default_rng(seed).integers(-128, 128, size=shape, dtype=np.int64).astype(np.int8)
        got = _run(native, native.ug_run_static, x)
        np.testing.assert_array_equal(got, golden_models[f"{name}/y{seed}"])
        np.testing.assert_array_equal(got, _run(native, native.ug_run, x))


def test_static_run_argument_checks(native, golden_ops):
    plan, x = golden_ops["add/plan"].tobytes(), golden_ops["add/x"]
    keep = _load(native, plan)  # noqa: F841
    y = np.empty(native.ug_output_bytes(), dtype=np.int8)
    assert native.ug_run_static(x.ctypes.data, x.nbytes - 1, y.ctypes.data, y.nbytes) == 22
    assert native.ug_run_static(None, x.nbytes, y.ctypes.data, y.nbytes) == 22
    assert native.ug_run_static(x.ctypes.data, x.nbytes, y.ctypes.data, y.nbytes) == 0  # still loaded
