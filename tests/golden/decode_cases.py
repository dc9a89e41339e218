"""Seeded inputs shared by tests/test_vision.py and make_decode_golden.py (no model files needed:
the YOLO contract is the bundled detector's metadata, restated here)."""
import base64

import numpy as np

PROFILE_TABLES = [((.485, .456, .406), (.229, .224, .225), .018249010667204857, -13, "|i1"),
                  ((0., 0., 0.), (1., 1., 1.), .003921568859368563, -128, "|i1"),
                  ((.5, .25, .125), (.3, .2, .1), .02, 7, "|u1")]
IMAGE_TABLES = [("|u1", (127.5,), (127.5,), 1 / 128, 128), ("|u1", (11., 127., 99.), (17., 64., 23.), .031, 13),
                ("|i1", (0.,), (255.,), 1 / 255, -128)]


def _image(seed, w, h):
    return np.random.default_rng(seed).integers(0, 256, size=(h, w, 3), dtype=np.int64).astype(np.uint8)


def profile_cases():
    crop = {"resize": "center_crop", "crop_pct": .875, "mean": [.485, .456, .406], "std": [.229, .224, .225]}
    box = {"resize": "letterbox", "mean": [0, 0, 0], "std": [1, 1, 1]}
    s224 = {"shape": (1, 224, 224, 3), "dtype": "int8", "quantization": {"scale": .018249010667204857, "zero_point": -13}}
    s320 = {"shape": (1, 320, 320, 3), "dtype": "int8", "quantization": {"scale": .003921568859368563, "zero_point": -128}}
    return [{"image": _image(1, 341, 199), "spec": s224, "profile": crop},
            {"image": _image(2, 180, 260), "spec": s224, "profile": crop},
            {"image": _image(3, 640, 427), "spec": s320, "profile": box},
            {"image": _image(4, 300, 500), "spec": s320, "profile": box}]


def image_cases():
    spec = {"shape": (1, 96, 128, 3), "dtype": np.dtype("i1"), "quantization": {"scale": 1 / 255, "zero_point": -128}}
    return [{"image": _image(5, 200, 150), "spec": spec, "normalization": {"mean": [0], "std": [255]}},
            {"image": _image(6, 64, 64), "spec": spec, "normalization": {"mean": [120, 110, 100], "std": [60, 58, 57]}}]


YOLO_QUANT = [(.03454255685210228, -105), (.16603389382362366, 117), (.05153468996286392, -126),
              (.7631877064704895, 124), (.04005463421344757, -128), (.4590281844139099, 120)]


def yolo_contract():
    names = [f"serving_default_output_{i}_output" for i in range(6)]
    outputs = []
    for i, stride in enumerate((8, 16, 32)):
        for j, c in ((0, 4), (1, 80)):
            k = 2 * i + j
            outputs.append({"name": names[k], "shape": (1, 320 // stride, 320 // stride, c), "dtype": "int8",
                            "quantization": {"scale": YOLO_QUANT[k][0], "zero_point": YOLO_QUANT[k][1]}})
    task = {"kind": "yolo_one_to_one", "schema": 1, "labels": [f"class{i}" for i in range(80)], "num_classes": 80,
            "strides": [8, 16, 32], "output_order": names}
    return task, outputs, (1, 320, 320, 3)


def yolo_cases(outputs):
    cases = []
    for seed in range(4):
        rng = np.random.default_rng(100 + seed)
        raw = {}
        for spec in outputs:
            if spec["shape"][-1] == 4:
                raw[spec["name"]] = rng.integers(-128, 128, size=spec["shape"]).astype(np.int8)
            else:  # mostly background logits with a few confident anchors
                v = rng.integers(-128, -60, size=spec["shape"]).astype(np.int16)
                hot = rng.random(spec["shape"]) < 0.004
                v[hot] = rng.integers(100, 128, size=int(hot.sum()))
                raw[spec["name"]] = v.astype(np.int8)
        geometry = {"ratio": .5 + .1 * seed, "left": 3 * seed, "top": 40 - 5 * seed, "width": 640, "height": 480}
        options = [{}, {"score_threshold": .1, "max_results": 50}, {"max_results": 5}, {"score_threshold": .9}][seed]
        cases.append((raw, geometry, options))
    return cases


def ssd_cases():
    cases = []
    for seed in range(3):
        rng = np.random.default_rng(200 + seed)
        n, c = 64, 3
        anchors = np.concatenate([rng.random((n, 2)), .05 + .3 * rng.random((n, 2))], axis=1).astype("<f4")
        task = {"kind": "ssd_fixed_anchors", "schema": 1, "num_boxes": n, "num_classes": c,
                "anchors_xywh_f32_base64": base64.b64encode(anchors.tobytes()).decode(),
                "scales_yxhw": [10., 10., 5., 5.], "exponential_size": seed != 1, "sigmoid_scores": seed == 2,
                "boxes_output": "boxes", "scores_output": "scores", "labels": ["a", "b", "c"]}
        raw = {"boxes": rng.normal(0, 2, size=(1, n, 4)).astype("f4"),
               "scores": (rng.random((1, n, c)) * (6 if seed == 2 else 1) - (3 if seed == 2 else 0)).astype("f4")}
        options = [{}, {"class_aware": True, "iou_threshold": .3}, {"score_threshold": .6, "max_results": 7}][seed]
        cases.append((task, raw, options))
    return cases


def pipeline_images(size):
    """Seeded RGB test images for whole-pipeline checks: smooth gradients with blocks, so the
    networks see structure rather than noise, in a few aspect ratios."""
    images = []
    for seed, (w, h) in enumerate([(size + 37, size - 21), (size - 40, size + 60), (2 * size, size)]):
        rng = np.random.default_rng(300 + seed)
        yy, xx = np.mgrid[:h, :w].astype("f4")
        img = np.stack([xx / w * 255, yy / h * 255, (xx + yy) / (w + h) * 255], axis=-1)
        for _ in range(6):
            x0, y0 = rng.integers(0, w - 20), rng.integers(0, h - 20)
            img[y0:y0 + rng.integers(10, h // 2), x0:x0 + rng.integers(10, w // 2)] = rng.integers(0, 256, 3)
        images.append(np.clip(img, 0, 255).astype(np.uint8))
    return images
