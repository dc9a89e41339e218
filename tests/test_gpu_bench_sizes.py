"""GPU parity at the batch sizes that are timed: MobileNetV4 at 256 and
4,096 images, YOLO26n at 128 and 1,024, through ug_infer_batch (host buffers, the copy/compute
pipeline from 512 images) and through the device-resident calls the bench times
(ug_upload_batch / ug_launch_batch / ug_download_batch). Every image at 256 / 128 and a strided
sample at 4,096 / 1,024 is compared byte for byte with the reference runtime's own output
(oracle/_ref/libug_ref.so, one image per call, run in a spawn pool: runtime/graph.c:438-448)."""
import ctypes as C

import numpy as np
import pytest

from conftest import model_path
from gpuhelp import NativeSession
from oracle.refpool import reference_outputs

pytestmark = pytest.mark.gpu
SHAPES = {"mobilenetv4-small": (224, 224, 3), "yolo26n-320": (320, 320, 3)}


def image(seed, index, shape):
    """Seeded image `index` of a batch: each image has its own stream, so any sample of a large
    batch can be regenerated without the rest."""
    return np.random.default_rng([seed, index]).integers(-128, 128, size=shape, dtype=np.int8)


def batch(seed, images, shape):
    return np.stack([image(seed, i, shape) for i in range(images)])


def sample(images, count):
    return sorted(set(np.linspace(0, images - 1, count).round().astype(int).tolist()))


@pytest.mark.parametrize("name,images", [("mobilenetv4-small", 256), ("yolo26n-320", 128)])
def test_every_image_of_a_timed_batch_matches_reference(name, images, native):
    from unoq_dsp import load
    plan = load(model_path(name)).plan
    xs = batch(21, images, SHAPES[name])
    expect = reference_outputs(plan, list(xs))
    with NativeSession(native, plan) as s:
        got = s.run(xs, images).reshape(images, -1)
    bad = [i for i in range(images) if not np.array_equal(got[i], expect[i])]
    assert not bad, f"{len(bad)} of {images} images differ, first {bad[:8]}"


@pytest.mark.parametrize("name,images,count", [("mobilenetv4-small", 4096, 12), ("yolo26n-320", 1024, 8)])
def test_bench_batch_device_resident_and_pipelined(name, images, count, native):
    """The bench's own batch sizes: the device-resident graph (the `value` path, replayed three times
    after one upload, so the input tensor must survive each replay) and the pipelined host batch
    (the `e2e` path) give identical outputs, and sampled images equal the reference's."""
    from unoq_dsp import load
    plan = load(model_path(name)).plan
    shape = SHAPES[name]
    xs = batch(22, images, shape)
    picks = sample(images, count)
    expect = reference_outputs(plan, [xs[i] for i in picks])
    with NativeSession(native, plan) as s:
        no = s.no
        h_in = native.ug_host_alloc(xs.nbytes)
        h_out = native.ug_host_alloc(no * images)
        try:
            C.memmove(h_in, xs.ctypes.data, xs.nbytes)
            assert native.ug_upload_batch(s.handle, h_in, images) == 0, native.ug_last_error()
            for _ in range(3):  # replays after one upload, as the bench times them
                assert native.ug_launch_batch(s.handle, images) == 0, native.ug_last_error()
            assert native.ug_synchronize(s.handle) == 0, native.ug_last_error()
            assert native.ug_download_batch(s.handle, h_out, images) == 0, native.ug_last_error()
            resident = np.ctypeslib.as_array(C.cast(h_out, C.POINTER(C.c_int8)), shape=(images, no)).copy()
            C.memset(h_out, 0, no * images)
            assert native.ug_infer_batch(s.handle, h_in, images, h_out) == 0, native.ug_last_error()
            piped = np.ctypeslib.as_array(C.cast(h_out, C.POINTER(C.c_int8)), shape=(images, no)).copy()
        finally:
            native.ug_host_free(h_in)
            native.ug_host_free(h_out)
    for j, i in enumerate(picks):
        np.testing.assert_array_equal(resident[i], expect[j], err_msg=f"device-resident image {i}")
    diff = np.flatnonzero((resident != piped).any(axis=1))
    assert diff.size == 0, f"pipelined batch differs from the device-resident one on images {diff[:8].tolist()}"


@pytest.mark.parametrize("case", ["block", "c2f_bytes", "transpose_nchw", "bmm_attn_qk"])
def test_replays_after_one_upload_keep_their_input(case, native, golden_ops):
    """ug_launch_batch replayed without a new upload gives the same bytes every time: no tensor of
    the step reuses the input tensor's storage."""
    plan, x = golden_ops[f"{case}/plan"].tobytes(), golden_ops[f"{case}/x"]
    images = 37
    rng = np.random.default_rng(8)
    xs = np.concatenate([x.reshape(1, -1)] + [rng.integers(-128, 128, size=(1, x.size), dtype=np.int64)
                                              .astype(np.int8) for _ in range(images - 1)])
    with NativeSession(native, plan) as s:
        expect = s.run(xs, images)
        assert native.ug_upload_batch(s.handle, xs.ctypes.data, images) == 0
        y = np.empty_like(expect)
        for _ in range(4):
            assert native.ug_launch_batch(s.handle, images) == 0
        assert native.ug_download_batch(s.handle, y.ctypes.data, images) == 0, native.ug_last_error()
    np.testing.assert_array_equal(y, expect)
    np.testing.assert_array_equal(y[:golden_ops[f"{case}/y"].size], golden_ops[f"{case}/y"])
