"""ug_infer_batch on large host batches: the copy/compute pipeline (pieces of the batch in two
alternating arena slots, H2D / compute / D2H on three streams) must give exactly the bytes of the
oracle for every image, including a short last piece, pinned and pageable host buffers alike."""
import ctypes as C

import numpy as np
import pytest

import opcases
from gpuhelp import NativeSession

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("images", [512, 777, 2101])
def test_pipelined_batch_matches_oracle(images, native, oracle):
    rng = np.random.default_rng(images)
    plan, x0 = opcases.block_case(rng, hw=7)
    xs = rng.integers(-128, 128, size=(images,) + x0.shape[1:], dtype=np.int64).astype(np.int8)
    expect = oracle.run(plan, xs, images)
    with NativeSession(native, plan) as s:
        np.testing.assert_array_equal(s.run(xs, images), expect)
        # pinned buffers, twice in a row (slots reused across calls)
        ni, no = s.ni * images, s.no * images
        hin, hout = native.ug_host_alloc(ni), native.ug_host_alloc(no)
        try:
            C.memmove(hin, xs.ctypes.data, ni)
            for _ in range(2):
                C.memset(hout, 0, no)
                assert native.ug_infer_batch(s.handle, hin, images, hout) == 0, native.ug_last_error()
                got = np.ctypeslib.as_array(C.cast(hout, C.POINTER(C.c_int8)), shape=(no,)).copy()
                np.testing.assert_array_equal(got, expect)
            assert native.ug_last_infer_ms(s.handle) > 0
        finally:
            native.ug_host_free(hin)
            native.ug_host_free(hout)


def test_pipeline_matches_single_piece_runs(native):
    """A pipelined batch equals the same images run as small (unpipelined) batches."""
    rng = np.random.default_rng(3)
    plan, x0 = opcases.block_case(rng, hw=7)
    images = 1030
    xs = rng.integers(-128, 128, size=(images,) + x0.shape[1:], dtype=np.int64).astype(np.int8)
    with NativeSession(native, plan) as s:
        piped = s.run(xs, images)
        step = 103
        parts = [s.run(xs[i:i + step], step) for i in range(0, images, step)]
    np.testing.assert_array_equal(piped, np.concatenate(parts))


def test_upload_launch_download_equals_host_batch(native):
    """Device-resident path (ug_upload_batch, ug_launch_batch, ug_download_batch) against the
    pipelined host call on the same images."""
    rng = np.random.default_rng(11)
    plan, x0 = opcases.block_case(rng, hw=7)
    images = 600
    xs = rng.integers(-128, 128, size=(images,) + x0.shape[1:], dtype=np.int64).astype(np.int8)
    with NativeSession(native, plan) as s:
        piped = s.run(xs, images)
        assert native.ug_upload_batch(s.handle, xs.ctypes.data, images) == 0
        assert native.ug_launch_batch(s.handle, images) == 0
        out = np.empty(s.no * images, np.int8)
        assert native.ug_download_batch(s.handle, out.ctypes.data, images) == 0
    np.testing.assert_array_equal(out, piped)
