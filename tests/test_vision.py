"""Host image preparation and box decoding (reference src/unoq_dsp/modern.py, vision.py) against
vectors produced by the reference package itself (tests/golden/make_decode_golden.py), plus
known-answer checks of the decoders. Exact equality: the float32 operation order is the same."""
import base64
import hashlib
import json
import sys
from pathlib import Path
from unittest.mock import patch

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import decode_cases as dc  # noqa: E402
from unoq_dsp import CompiledModel, ImageClassifier  # noqa: E402
from unoq_dsp.errors import UnsupportedModel  # noqa: E402
from unoq_dsp.modern import YOLODecoder, prepare_profile, profile_lookup  # noqa: E402
from unoq_dsp.vision import SSDDecoder, image_lookup, prepare_image  # noqa: E402

GOLD = json.loads((Path(__file__).resolve().parent / "golden" / "decode.json").read_text())


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def flat(detections):
    return [[d.class_id, d.label, d.score, list(d.box)] for d in detections]


def test_lookup_tables_match_reference():
    assert [sha(profile_lookup(*a)) for a in dc.PROFILE_TABLES] == GOLD["profile_lookup"]
    assert [sha(image_lookup(*a)) for a in dc.IMAGE_TABLES] == GOLD["image_lookup"]


def test_prepare_profile_matches_reference():
    got = []
    for case in dc.profile_cases():
        x, geometry = prepare_profile(case["image"], case["spec"], case["profile"])
        got.append([sha(x), geometry])
    assert got == GOLD["prepare_profile"]


def test_prepare_image_matches_reference():
    got = [[sha(x), list(size)] for x, size in
           (prepare_image(c["image"], c["spec"], c["normalization"]) for c in dc.image_cases())]
    assert got == GOLD["prepare_image"]


def test_yolo_decode_matches_reference():
    task, outputs, shape = dc.yolo_contract()
    decoder = YOLODecoder(task, outputs, shape)
    got = [flat(decoder.decode(raw, geometry=g, **o)) for raw, g, o in dc.yolo_cases(outputs)]
    assert got == GOLD["yolo"]
    assert sum(map(len, got)) > 50  # the cases do produce detections


def test_ssd_decode_matches_reference():
    assert [flat(SSDDecoder(t).decode(raw, **o)) for t, raw, o in dc.ssd_cases()] == GOLD["ssd"]


# ---- known answers (constructed by hand) ---------------------------------------------------

def ssd_task():
    anchors = np.array([[.5, .5, .4, .2], [.5, .5, .4, .2], [.1, .1, .1, .1]], dtype="<f4")
    task = {"kind": "ssd_fixed_anchors", "schema": 1, "num_boxes": 3, "num_classes": 2,
            "anchors_xywh_f32_base64": base64.b64encode(anchors.tobytes()).decode(), "scales_yxhw": [1, 1, 1, 1],
            "exponential_size": True, "sigmoid_scores": False, "boxes_output": "boxes", "scores_output": "scores",
            "labels": ["person", "cat"]}
    outputs = {"boxes": np.zeros((1, 3, 4), "f4"), "scores": np.array([[[.9, .1], [.1, .85], [.7, .2]]], "f4")}
    return task, outputs


def test_ssd_zero_offsets_give_the_anchor_and_nms_suppresses_the_duplicate():
    task, outputs = ssd_task()
    d = SSDDecoder(task).decode(outputs)
    assert [x.label for x in d] == ["person", "person"]  # anchor 1 (cat) overlaps anchor 0 fully
    np.testing.assert_allclose(d[0].box, [.3, .4, .7, .6], atol=1e-7)
    np.testing.assert_allclose(d[1].box, [.05, .05, .15, .15], atol=1e-7)
    assert [x.label for x in SSDDecoder(task).decode(outputs, class_aware=True)] == ["person", "cat", "person"]
    assert SSDDecoder(task).decode(outputs, score_threshold=.99) == []
    with pytest.raises(ValueError):
        SSDDecoder(task).decode(outputs, iou_threshold=float("nan"))
    outputs["boxes"][0, 0, 0] = np.nan
    with pytest.raises(ValueError):
        SSDDecoder(task).decode(outputs)


def tiny_yolo():
    names = [f"o{i}" for i in range(6)]
    specs, outputs = [], {}
    for i, stride in enumerate((8, 16, 32)):
        h = 64 // stride
        for j, c in ((0, 4), (1, 2)):
            spec = {"name": names[2 * i + j], "shape": (1, h, h, c), "dtype": "int8",
                    "quantization": {"scale": .125 if j == 0 else .25, "zero_point": 0}}
            specs.append(spec)
            outputs[spec["name"]] = np.full(spec["shape"], 8 if j == 0 else -100, "i1")
    task = {"kind": "yolo_one_to_one", "schema": 1, "labels": ["a", "b"], "num_classes": 2, "strides": [8, 16, 32],
            "output_order": names}
    return YOLODecoder(task, specs, (1, 64, 64, 3)), outputs


def test_yolo_grid_decode_and_inverse_letterbox():
    decoder, outputs = tiny_yolo()
    outputs["o1"][0, 2, 3, 1] = 8  # logit 2.0 for class b at cell (x=3, y=2) of stride 8
    d = decoder.decode(outputs, geometry={"ratio": .5, "left": 0, "top": 16, "width": 128, "height": 64})
    assert len(d) == 1 and d[0].label == "b"
    assert d[0].score == pytest.approx(1 / (1 + np.exp(-2)), abs=1e-6)
    # centre (3.5, 2.5) +- 1 cell, x8 -> (20, 12, 36, 28) px; undo the letterbox, clip to [0, 1]
    np.testing.assert_allclose(d[0].box, (20 / 64, max(0, (12 - 16) / 32), 36 / 64, (28 - 16) / 32), atol=1e-7)


def test_yolo_classes_share_an_anchor_and_arguments_are_checked():
    decoder, outputs = tiny_yolo()
    outputs["o1"][0, 2, 3] = [8, 7]
    d = decoder.decode(outputs, geometry={"ratio": 1, "left": 0, "top": 0, "width": 64, "height": 64})
    assert [x.class_id for x in d] == [0, 1] and d[0].box == d[1].box
    with pytest.raises(ValueError):
        decoder.decode(outputs, geometry={}, score_threshold=1.2)
    with pytest.raises(ValueError):
        decoder.decode(outputs, geometry={}, iou_threshold=.5)
    with pytest.raises(UnsupportedModel):
        YOLODecoder({"kind": "yolo_one_to_one", "schema": 2}, [], (1, 64, 64, 3))


def test_classifier_uses_dequantised_output_once():
    spec = {"shape": (1, 1, 1, 3), "dtype": np.dtype("i1"), "quantization": {"scale": 1 / 255, "zero_point": -128}}
    output = {"shape": (1, 2), "dtype": np.dtype("i1"), "quantization": {"scale": 1 / 256, "zero_point": -128},
              "dequantize": True}
    model = CompiledModel(b"", {"input": spec, "output": output, "outputs": [output]})
    with patch("unoq_dsp.vision.Session") as session:
        session.return_value.metadata = model.metadata
        session.return_value.run.return_value = np.array([[.125, .875]], "f4")
        with ImageClassifier(model, mean=[0], std=[255], labels=["a", "b"]) as classifier:
            assert classifier.classify(np.zeros((1, 1, 3), "u1"), top_k=1) == [{"class_id": 1, "label": "b",
                                                                                  "score": .875}]
