"""GPU parity on the two bundled models (BASELINE configs 2/3): raw int8 outputs bit-exact
with the reference runtime, at batch 1 and in batches, through the C ABI and the Python API."""
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import model_path
from gpuhelp import NativeSession

pytestmark = pytest.mark.gpu
MODELS = [("mobilenetv4-small", (1, 224, 224, 3)), ("yolo26n-320", (1, 320, 320, 3))]


def seeded(shape, seed):
    return np.random.default_rng(seed).integers(-128, 128, size=shape, dtype=np.int64).astype(np.int8)


@pytest.mark.parametrize("name,shape", MODELS)
def test_batch1_matches_reference_golden(name, shape, native, golden_models):
    from unoq_dsp import load
    model = load(model_path(name))
    with NativeSession(native, model.plan) as s:
        for seed in (0, 1):
            np.testing.assert_array_equal(s.run(seeded(shape, seed)), golden_models[f"{name}/y{seed}"])


@pytest.mark.parametrize("name,shape", MODELS)
def test_batch_matches_oracle(name, shape, native, oracle):
    from unoq_dsp import load
    model = load(model_path(name))
    images = 5
    xs = np.concatenate([seeded(shape, 100 + i) for i in range(images)])
    expect = oracle.run(model.plan, xs, images)
    with NativeSession(native, model.plan) as s:
        np.testing.assert_array_equal(s.run(xs, images), expect)


@pytest.mark.parametrize("name,shape", MODELS)
def test_large_batch_is_image_independent(name, shape, native):
    """Size-independent property at a large batch: every image's output equals the output of
    that image run alone (the batched arena never couples images)."""
    from unoq_dsp import load
    model = load(model_path(name))
    images = 64
    xs = np.concatenate([seeded(shape, 500 + i) for i in range(images)])
    with NativeSession(native, model.plan) as s:
        got = s.run(xs, images).reshape(images, -1)
        for i in (0, 17, 63):
            np.testing.assert_array_equal(got[i], s.run(xs[i:i + 1]))


def test_python_session_unpacks_yolo_outputs(golden_models):
    from unoq_dsp import Session, load
    model = load(model_path("yolo26n-320"))
    x = seeded((1, 320, 320, 3), 0)
    with Session(model) as s:
        outputs = s.run(x)
        batch = s.run_batch(np.concatenate([x, x]))
    wire = golden_models["yolo26n-320/y0"].view(np.uint8)
    for spec in model.metadata["outputs"]:
        lo = spec["packed_offset"]
        ref = wire[lo:lo + spec["bytes"]].view(spec["dtype"]).reshape(spec["shape"])
        np.testing.assert_array_equal(outputs[spec["name"]], ref)
        np.testing.assert_array_equal(batch[1][spec["name"]], ref)


# ---- whole pipelines through the public Python API ------------------------------------------

def _decode_gold():
    import json
    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    import decode_cases
    return decode_cases, json.loads((Path(__file__).resolve().parent / "golden" / "decode.json").read_text())


def test_image_classifier_matches_reference_pipeline():
    """ImageClassifier (bundled center-crop profile, softmax, top-5) on the GPU against the
    reference's ImageClassifier driven by the reference runtime, on seeded images."""
    from unoq_dsp import ImageClassifier
    dc, gold = _decode_gold()
    with ImageClassifier(model_path("mobilenetv4-small")) as clf:
        got = [[[r["class_id"], r["label"], r["score"]] for r in clf.classify(im, top_k=5)]
               for im in dc.pipeline_images(224)]
        batch = clf.classify_batch(dc.pipeline_images(224), top_k=5)
    assert got == gold["classify"]
    assert [[[r["class_id"], r["label"], r["score"]] for r in res] for res in batch] == gold["classify"]


def test_object_detector_matches_reference_pipeline():
    """ObjectDetector (letterbox, six packed int8 heads, one-to-one decode) on the GPU: boxes and
    scores identical to the reference pipeline's."""
    from unoq_dsp import ObjectDetector
    dc, gold = _decode_gold()
    flat = lambda ds: [[d.class_id, d.label, d.score, list(d.box)] for d in ds]  # noqa: E731
    with ObjectDetector(model_path("yolo26n-320")) as det:
        got = [flat(det.detect(im, score_threshold=0.0, max_results=30)) for im in dc.pipeline_images(320)]
        batch = det.detect_batch(dc.pipeline_images(320), score_threshold=0.0, max_results=30)
    assert got == gold["detect"]
    assert [flat(b) for b in batch] == gold["detect"]


def test_models_identical_with_and_without_add_fusion(native, golden_models, monkeypatch):
    """Both bundled models with residual adds fused into conv epilogues and with separate adds."""
    from unoq_dsp import load
    for name, shape in MODELS:
        plan = load(model_path(name)).plan
        x = seeded(shape, 0)
        with NativeSession(native, plan) as s:
            fused = s.run(x)
        monkeypatch.setenv("UNOQ_FUSE_ADD", "0")
        with NativeSession(native, plan) as s:
            separate = s.run(x)
        monkeypatch.delenv("UNOQ_FUSE_ADD")
        np.testing.assert_array_equal(fused, golden_models[f"{name}/y0"])
        np.testing.assert_array_equal(separate, golden_models[f"{name}/y0"])
