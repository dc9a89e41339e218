"""ug_run_static, the allocation-free variant of ug_run (fixed 16 MiB device arena, direct
launches), against ug_run on the same graph: identical bytes on two calls in a row, with
ug_run interleaved, for op plans and both bundled models; snapshots of intermediate tensors after
either call; and device memory that does not move across calls once the set-up call is done.
Collected last on purpose: it must pass alone and after every other test of the session."""
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


def _intermediates(plan, limit=4):
    """Intermediate activations that every run writes: depthwise outputs (a conv's output that
    feeds a residual add may be left unwritten, the add being computed in the conv's epilogue)."""
    import struct
    magic, version, nt, no, arena, inp, out, flags = struct.unpack_from("<8I", plan)
    ts = [struct.unpack_from("<12I", plan, 32 + 48 * i) for i in range(nt)]
    ops = [struct.unpack_from("<8I", plan, 32 + 48 * nt + 32 * i) for i in range(no)]
    seen = []
    for o in ops:
        z = o[3]
        if o[0] == 15 and z not in (inp, out) and not ts[z][8] and z not in seen:
            seen.append(z)
    step = max(1, len(seen) // limit)
    return [(t, ts[t][1]) for t in seen[::step][:limit]]


def _snap(native, tensor, size):
    buf = np.empty(size, dtype=np.int8)
    assert native.ug_snapshot(tensor, buf.ctypes.data, size) == 0, native.ug_last_error()
    return buf


def test_static_run_snapshots_its_own_arena(native):
    """ug_snapshot after ug_run_static reads the static arena: it equals the snapshot after ug_run
    of the same input (both runs lay the one-image plan out identically), and it follows the input."""
    from unoq_dsp import load
    plan = load(model_path("mobilenetv4-small")).plan
    keep = _load(native, plan)  # noqa: F841
    rng = np.random.default_rng(11)
    xa, xb = (rng.integers(-128, 128, size=224 * 224 * 3, dtype=np.int64).astype(np.int8) for _ in range(2))
    picks = _intermediates(plan)
    assert picks
    _run(native, native.ug_run, xa)
    after_run = [_snap(native, t, n) for t, n in picks]
    _run(native, native.ug_run_static, xb)  # a different image through the static arena
    _run(native, native.ug_run_static, xa)
    after_static = [_snap(native, t, n) for t, n in picks]
    for (t, _), a, b in zip(picks, after_run, after_static):
        np.testing.assert_array_equal(a, b, err_msg=f"tensor {t}")


def test_static_run_allocates_no_device_memory(native):
    """After the set-up call, repeated ug_run_static calls leave the device's free memory unchanged
    (any cudaMalloc, even of a few bytes, takes at least one 2 MiB page from the device)."""
    torch = pytest.importorskip("torch")
    from unoq_dsp import load
    plan = load(model_path("yolo26n-320")).plan
    keep = _load(native, plan)  # noqa: F841
    x = np.random.default_rng(3).integers(-128, 128, size=320 * 320 * 3, dtype=np.int64).astype(np.int8)
    first = _run(native, native.ug_run_static, x)  # set-up call
    torch.cuda.synchronize()
    free_before, _ = torch.cuda.mem_get_info(0)
    for _ in range(3):
        np.testing.assert_array_equal(_run(native, native.ug_run_static, x), first)
    free_after, _ = torch.cuda.mem_get_info(0)
    assert free_after == free_before, (free_before, free_after)
