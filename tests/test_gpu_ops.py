"""GPU parity, per opcode: libunoq_cuda.so through its C ABI against the reference's outputs
(golden fixtures) and against the oracle at larger sizes and batches. Bit-exact throughout:
every op is integer arithmetic."""
import ctypes as C

import numpy as np
import pytest

import opcases
from gpuhelp import NativeSession

pytestmark = pytest.mark.gpu
NAMES = [n for n, _ in opcases.all_cases(1)]


@pytest.mark.parametrize("name", NAMES)
def test_graph_abi_matches_reference_golden(name, native, golden_ops):
    """ug_load + ug_run (runtime/graph.h ABI), one image, against the reference runtime's output."""
    plan = golden_ops[f"{name}/plan"].tobytes()
    x = golden_ops[f"{name}/x"]
    buf = C.create_string_buffer(plan, len(plan))
    assert native.ug_load(buf, len(plan)) == 0, native.ug_last_error()
    no = native.ug_output_bytes()
    y = np.empty(no, dtype=np.int8)
    assert native.ug_run(x.ctypes.data, x.nbytes, y.ctypes.data, no) == 0, native.ug_last_error()
    np.testing.assert_array_equal(y, golden_ops[f"{name}/y"])


@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("images", [3])
def test_batched_session_matches_oracle_at_scale(name, images, native, oracle):
    builder = dict(opcases.all_cases(4))[name]
    rng = np.random.default_rng(101)
    plan, x0 = builder(rng)
    xs = np.stack([x0] + [rng.integers(-128, 128, size=x0.shape, dtype=np.int64).astype(np.int8)
                          for _ in range(images - 1)])
    expect = oracle.run(plan, xs, images)
    with NativeSession(native, plan) as s:
        got = s.run(xs, images)
        np.testing.assert_array_equal(got, expect)
        # the same images one at a time give the same bytes (no cross-image coupling)
        single = s.run(xs[1])
        np.testing.assert_array_equal(single, expect[single.size:2 * single.size])


def test_reload_replaces_graph(native, golden_ops):
    for name in ("conv_pw_c0", "dw3_s2", "softmax_exact"):
        plan = golden_ops[f"{name}/plan"].tobytes()
        assert native.ug_load(C.create_string_buffer(plan, len(plan)), len(plan)) == 0
    assert native.ug_output_bytes() == golden_ops["softmax_exact/y"].size


def test_bad_calls_return_reference_codes(native, golden_ops):
    plan = golden_ops["add/plan"].tobytes()
    assert native.ug_load(C.create_string_buffer(plan, len(plan)), len(plan)) == 0
    x = golden_ops["add/x"]
    y = np.empty(golden_ops["add/y"].size, dtype=np.int8)
    assert native.ug_run(x.ctypes.data, x.nbytes - 1, y.ctypes.data, y.nbytes) == 22
    assert native.ug_snapshot(0, y.ctypes.data, 3) == 22
    err = C.c_int()
    h = native.ug_open_mode(C.create_string_buffer(plan, len(plan)), len(plan), 0, C.byref(err))
    assert h and err.value == 0
    h2 = native.ug_open_mode(C.create_string_buffer(plan, len(plan)), len(plan), 0, C.byref(err))
    assert not h2 and err.value == 1001  # one session per process (bridge.c:101)
    assert native.ug_infer(h, x.ctypes.data, x.nbytes + 1, y.ctypes.data, y.nbytes) == 1003
    native.ug_close(h)
    native.ug_close(None)


def test_snapshot_and_profile(native, golden_ops):
    plan = golden_ops["block/plan"].tobytes()
    assert native.ug_load(C.create_string_buffer(plan, len(plan)), len(plan)) == 0
    counters = np.zeros(514, dtype=np.uint64)
    assert native.ug_profile(1, counters.ctypes.data, counters.nbytes) == 0
    x = golden_ops["block/x"]
    y = np.empty(golden_ops["block/y"].size, dtype=np.int8)
    assert native.ug_run(x.ctypes.data, x.nbytes, y.ctypes.data, y.nbytes) == 0
    np.testing.assert_array_equal(y, golden_ops["block/y"])
    assert native.ug_profile(2, counters.ctypes.data, counters.nbytes) == 0
    assert counters[0] == 1 and counters[1] > 0
    inp = np.empty(x.size, dtype=np.int8)
    assert native.ug_snapshot(0, inp.ctypes.data, inp.nbytes) == 0
    np.testing.assert_array_equal(inp, x)


@pytest.mark.parametrize("name", ["block", "block_conv_second"])
def test_fused_residual_add_matches_unfused(name, native, oracle, monkeypatch):
    """A residual add computed in the projection conv's epilogue gives the bytes of the separate
    add kernel (UNOQ_FUSE_ADD=0) and of the oracle, at batch 1 and in a batch."""
    rng = np.random.default_rng(17)
    plan, x0 = dict(opcases.all_cases(2))[name](rng)
    xs = np.stack([x0] + [rng.integers(-128, 128, size=x0.shape, dtype=np.int64).astype(np.int8) for _ in range(5)])
    expect = oracle.run(plan, xs, 6)
    with NativeSession(native, plan) as s:
        fused = s.run(xs, 6)
    monkeypatch.setenv("UNOQ_FUSE_ADD", "0")
    with NativeSession(native, plan) as s:
        separate = s.run(xs, 6)
    np.testing.assert_array_equal(fused, expect)
    np.testing.assert_array_equal(separate, expect)


@pytest.mark.parametrize("x_shape,oc,stride", [((1, 300, 48, 3), 16, (2, 2)), ((1, 131, 64, 3), 32, (1, 1)),
                                               ((1, 224, 224, 3), 32, (2, 2))])
def test_row_gemm_conv_tiles_and_edges(native, oracle, monkeypatch, x_shape, oc, stride):
    """The few-channel row-GEMM conv over more than one 128-row tile per image and a partial last
    column group, against the oracle and against the same plan with that path switched off."""
    from unoq_dsp import synth
    rng = np.random.default_rng(sum(x_shape) + oc)
    plan, xs, _ = synth.single_conv_plan(rng, x_shape, oc, (3, 3), stride, xq=(0.02, -9))
    images = 3
    x = rng.integers(-128, 128, size=(images,) + xs[1:], dtype=np.int64).astype(np.int8)
    expect = oracle.run(plan, x, images)
    with NativeSession(native, plan) as s:
        np.testing.assert_array_equal(s.run(x, images), expect)
    monkeypatch.setenv("UNOQ_CONV_ROWS", "0")
    with NativeSession(native, plan) as s:
        np.testing.assert_array_equal(s.run(x, images), expect)


@pytest.mark.parametrize("padding", ["same", (2, 0, 1, 3)])
def test_gather_mode_conv_wide_rows(native, oracle, padding):
    """Input rows too wide for the band path (32 KB each) take the tensor-core conv's per-tap
    gather, whose taps outside the image are written as the zero point directly."""
    from unoq_dsp import synth
    rng = np.random.default_rng(77)
    plan, xs, _ = synth.single_conv_plan(rng, (1, 9, 512, 64), 32, (3, 3), (1, 1), xq=(0.02, 21), padding=padding)
    images = 2
    x = rng.integers(-128, 128, size=(images,) + xs[1:], dtype=np.int64).astype(np.int8)
    with NativeSession(native, plan) as s:
        np.testing.assert_array_equal(s.run(x, images), oracle.run(plan, x, images))


TAP_CASES = [n for n in NAMES if n.startswith("conv_taps") or n in ("conv_3x3_s1", "conv_3x3_s2", "conv_wide_k",
                                                                      "conv_post_lut")]


@pytest.mark.parametrize("name", TAP_CASES)
def test_tap_tma_conv_on_every_eligible_case(name, native, golden_ops, monkeypatch):
    """The per-tap TMA conv (taken by default only for 128-byte channel chunks) on every op case
    with ic % 32 == 0: 32 / 64 / 128-byte chunks, dilation, odd sizes, post table."""
    monkeypatch.setenv("UNOQ_CONV_TAPS", "all")
    plan = golden_ops[f"{name}/plan"].tobytes()
    x = golden_ops[f"{name}/x"]
    with NativeSession(native, plan) as s:
        np.testing.assert_array_equal(s.run(x), golden_ops[f"{name}/y"])
