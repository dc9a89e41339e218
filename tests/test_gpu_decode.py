"""GPU: on-device preparation and decoding (include/unoq_cuda.h ug_set_input_table,
ug_set_yolo_decode, ug_detect_batch) on the bundled models. The decoder's records must equal the
numpy restatement of its contract (tests/decode_emulation.py) bit for bit on the network's own
outputs, and the image APIs must give identical results with on_device=True and False."""
import ctypes as C
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import model_path
from decode_emulation import emulate
from gpuhelp import NativeSession

pytestmark = pytest.mark.gpu
sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))


def yolo():
    from unoq_dsp.bundle import load
    from unoq_dsp.modern import YOLODecoder
    model = load(model_path("yolo26n-320"))
    md = model.metadata
    return model, YOLODecoder(md["task"], md["outputs"], md["input"]["shape"])


def seeded(n, shape, seed):
    return np.random.default_rng(seed).integers(-128, 128, size=(n,) + shape[1:], dtype=np.int64).astype(np.int8)


def detect(native, handle, x, k):
    from unoq_dsp.native import RECORD_DTYPE
    rec = np.empty((len(x), k), dtype=RECORD_DTYPE)
    rc = native.ug_detect_batch(handle, x.ctypes.data, len(x), k, rec.ctypes.data)
    assert rc == 0, native.ug_last_error()
    return rec


@pytest.mark.parametrize("images,k", [(1, 20), (7, 300), (64, 1), (33, 512), (600, 100)])
def test_records_match_the_decoder_contract(native, images, k):
    """600 images run through the pipelined (pieces) path."""
    model, decoder = yolo()
    config = decoder.device_config()
    x = seeded(images, (1, 320, 320, 3), images)
    with NativeSession(native, model.plan) as s:
        assert native.ug_set_yolo_decode(s.handle, C.byref(config)) == 0, native.ug_last_error()
        got = detect(native, s.handle, x, k)
        raw = s.run(x, images).reshape(images, -1)
    want = emulate(config, raw, k)
    assert got.tobytes() == want.tobytes()


def test_input_table_equals_host_lookup(native):
    from unoq_dsp.modern import profile_lookup
    model, decoder = yolo()
    table = profile_lookup((0.0, 0.0, 0.0), (1.0, 1.0, 1.0), model.metadata["input"]["quantization"]["scale"],
                           model.metadata["input"]["quantization"]["zero_point"], "|i1")
    pixels = np.random.default_rng(9).integers(0, 256, size=(5, 320, 320, 3), dtype=np.uint8)
    host = table[pixels, np.arange(3)]
    config = decoder.device_config()
    with NativeSession(native, model.plan) as s:
        assert native.ug_set_yolo_decode(s.handle, C.byref(config)) == 0
        plain_raw = s.run(host, 5)
        plain_rec = detect(native, s.handle, host, 50)
        t = np.ascontiguousarray(table)
        assert native.ug_set_input_table(s.handle, t.ctypes.data, 3) == 0, native.ug_last_error()
        np.testing.assert_array_equal(s.run(pixels, 5), plain_raw)
        assert detect(native, s.handle, pixels, 50).tobytes() == plain_rec.tobytes()
        assert native.ug_set_input_table(s.handle, None, 0) == 0
        np.testing.assert_array_equal(s.run(host, 5), plain_raw)


def test_classifier_input_table_at_scale(native):
    """A batch large enough for the pipelined path, through the byte table on the GPU."""
    from unoq_dsp.bundle import load
    from unoq_dsp.modern import profile_lookup
    model = load(model_path("mobilenetv4-small"))
    q = model.metadata["input"]["quantization"]
    prof = model.metadata["task"]["preprocessing"]
    table = np.ascontiguousarray(profile_lookup(tuple(prof["mean"]), tuple(prof["std"]), q["scale"], q["zero_point"],
                                                "|i1"))
    pixels = np.random.default_rng(3).integers(0, 256, size=(700, 224, 224, 3), dtype=np.uint8)
    with NativeSession(native, model.plan) as s:
        want = s.run(table[pixels, np.arange(3)], 700)
        assert native.ug_set_input_table(s.handle, table.ctypes.data, 3) == 0
        np.testing.assert_array_equal(s.run(pixels, 700), want)


def test_decoder_arguments_are_checked(native):
    from unoq_dsp.native import RECORD_DTYPE
    model, decoder = yolo()
    x = seeded(1, (1, 320, 320, 3), 0)
    rec = np.empty((1, 4), dtype=RECORD_DTYPE)
    with NativeSession(native, model.plan) as s:
        assert native.ug_detect_batch(s.handle, x.ctypes.data, 1, 4, rec.ctypes.data) == 1003  # no decoder yet
        for field, value in (("levels", 0), ("classes", 0), ("candidates", 513), ("reserved", 1)):
            bad = decoder.device_config()
            setattr(bad, field, value)
            assert native.ug_set_yolo_decode(s.handle, C.byref(bad)) == 1003, field
        bad = decoder.device_config()
        bad.level[2].score_offset = 176400 - 10  # the level's logits would run past the output
        assert native.ug_set_yolo_decode(s.handle, C.byref(bad)) == 1003
        bad = decoder.device_config()
        bad.level[0].rank[5] = 1024
        assert native.ug_set_yolo_decode(s.handle, C.byref(bad)) == 1003
        good = decoder.device_config()
        assert native.ug_set_yolo_decode(s.handle, C.byref(good)) == 0
        for k in (0, 513):
            assert native.ug_detect_batch(s.handle, x.ctypes.data, 1, k, rec.ctypes.data) == 1003
        t = np.zeros((256, 17), np.int8)
        assert native.ug_set_input_table(s.handle, t.ctypes.data, 7) == 1003   # 7 does not divide 320*320*3
        assert native.ug_set_input_table(s.handle, t.ctypes.data, 17) == 1003
        assert native.ug_set_yolo_decode(s.handle, None) == 0
        assert native.ug_detect_batch(s.handle, x.ctypes.data, 1, 4, rec.ctypes.data) == 1003


def _images(n, seed):
    rng = np.random.default_rng(seed)
    out = []
    for i in range(n):
        h, w = rng.integers(180, 700, size=2)
        img = rng.integers(0, 256, size=(h, w, 3), dtype=np.uint8)
        img[: h // 2] = (np.arange(w)[None, :, None] * (i + 1)) % 256  # structure in half the image
        out.append(img)
    return out


def test_object_detector_on_device_equals_host():
    from unoq_dsp import ObjectDetector
    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    import decode_cases as dc
    images = dc.pipeline_images(320) + _images(6, 1)
    grid = [{}, {"score_threshold": 0.0, "max_results": 300}, {"score_threshold": 0.05, "max_results": 7}]
    results = {}
    for on_device in (True, False):
        with ObjectDetector(model_path("yolo26n-320"), on_device=on_device) as det:
            assert det.device_decode is on_device
            results[on_device] = ([[det.detect(im, **o) for im in images] for o in grid],
                                  [det.detect_batch(images, **o) for o in grid])
    assert results[True] == results[False]
    assert sum(len(d) for d in results[True][0][1]) > 300


def test_image_classifier_on_device_equals_host():
    from unoq_dsp import ImageClassifier
    images = _images(5, 2)
    results = {}
    for on_device in (True, False):
        with ImageClassifier(model_path("mobilenetv4-small"), on_device=on_device) as clf:
            results[on_device] = ([clf.classify(im, top_k=10) for im in images], clf.classify_batch(images, top_k=3))
    assert results[True] == results[False]
