"""Image APIs: network on the GPU, explicit host image preparation and box decoding.

The reference's src/unoq_dsp/vision.py surface: ``ImageClassifier.classify``,
``ObjectDetector.detect``, ``Detection``, ``SSDDecoder`` (fixed anchors + NMS), ``prepare_image``
and ``image_lookup``. Float32 arithmetic follows the reference's operation order, so labels,
scores and boxes are identical for identical int8 network outputs. The batch methods
(``classify_batch``, ``detect_batch``) are this backend's extension: one GPU call for N images,
then the same per-image decoding.

With ``on_device=True`` (the default) the byte table runs on the GPU (the host only resizes and
uploads uint8 pixels), and the one-to-one YOLO decoder's top-k runs on the GPU too, returning a
few records per image instead of the raw head outputs; ``on_device=False`` keeps the table and
the decoding on the host. Both give identical results.
"""
import base64
import time
from dataclasses import dataclass
from functools import lru_cache
from pathlib import Path

import numpy as np

from . import CompiledModel, Session, compile_model, load
from .errors import UnsupportedModel


def resolve(model):
    if isinstance(model, CompiledModel):
        return model
    return load(model) if Path(model).suffix == ".uqmodel" else compile_model(model)


@lru_cache(maxsize=64)
def image_lookup(dtype, mean, std, scale, zero):
    """256x3 table: byte -> round-half-away((b - mean) / std / scale) + zero, clipped (vision.py:20-29)."""
    scaled = (np.arange(256, dtype="f4")[:, None] - np.asarray(mean, dtype="f4")) / np.asarray(std, dtype="f4") \
        / np.float32(scale)
    rounded = np.where(scaled >= 0, np.floor(scaled + .5), np.ceil(scaled - .5)) + np.float32(zero)
    info = np.iinfo(dtype)
    table = np.broadcast_to(np.clip(rounded, info.min, info.max), (256, 3)).astype(dtype)
    table.flags.writeable = False
    return table


def prepare_image(image, spec, normalization):
    """Bilinear resize to the input shape, then the lookup table (vision.py:32-51)."""
    pixels, table, size = image_pixels(image, spec, normalization)
    return table[pixels[0], np.arange(3)][None], size


def image_pixels(image, spec, normalization):
    """``prepare_image`` before its table lookup: ((1, H, W, 3) uint8 pixels, (256, 3) table, size)."""
    from PIL import Image
    if isinstance(image, np.ndarray):
        if image.dtype != np.uint8 or image.ndim != 3 or image.shape[2] != 3:
            raise ValueError("Expected an H×W×3 uint8 RGB image")
        image = Image.fromarray(image)
    if not isinstance(image, Image.Image):
        raise TypeError("Pass a Pillow image or uint8 RGB array")
    shape = tuple(spec["shape"])
    if len(shape) != 4 or shape[0] != 1 or shape[3] != 3:
        raise UnsupportedModel("Image API requires batch-one NHWC RGB input")
    mean = np.asarray(normalization["mean"], dtype="f4")
    std = np.asarray(normalization["std"], dtype="f4")
    if mean.size not in (1, 3) or std.size not in (1, 3) or not np.all(np.isfinite(mean)) \
            or not np.all(np.isfinite(std)) or np.any(std <= 0):
        raise ValueError("Expected finite RGB normalization with positive standard deviations")
    pixels = np.asarray(image.convert("RGB").resize((shape[2], shape[1]), Image.Resampling.BILINEAR), dtype="u1")
    q = spec["quantization"]
    table = image_lookup(np.dtype(spec["dtype"]).str, tuple(float(v) for v in mean.reshape(-1)),
                         tuple(float(v) for v in std.reshape(-1)), q["scale"], q["zero_point"])
    return pixels[None], table, image.size


@dataclass(frozen=True)
class Detection:
    class_id: int
    label: str
    score: float
    box: tuple  # normalised x_min, y_min, x_max, y_max in the original image


class SSDDecoder:
    """Fixed-anchor SSD head: anchor decode, score threshold, greedy NMS (vision.py:62-132)."""

    def __init__(self, task):
        if task.get("kind") != "ssd_fixed_anchors" or task.get("schema") != 1:
            raise UnsupportedModel("No supported fixed-anchor detector task metadata")
        self.task = task
        self.count, self.classes = task["num_boxes"], task["num_classes"]
        if type(self.count) is not int or type(self.classes) is not int or not 1 <= self.count <= 100000 \
                or not 1 <= self.classes <= 4096:
            raise UnsupportedModel("Invalid detector dimensions")
        encoded = task["anchors_xywh_f32_base64"]
        if not isinstance(encoded, str) or len(encoded) > ((self.count * 16 + 2) // 3) * 4:
            raise UnsupportedModel("Invalid anchor payload length")
        raw = base64.b64decode(encoded, validate=True)
        if len(raw) != self.count * 16:
            raise UnsupportedModel("Invalid anchor count")
        self.anchors = np.frombuffer(raw, dtype="<f4").reshape(self.count, 4)
        self.scales = np.asarray(task["scales_yxhw"], dtype="f4")
        if self.scales.shape != (4,) or not np.all(np.isfinite(self.scales)) or np.any(self.scales <= 0) \
                or not np.all(np.isfinite(self.anchors)) or np.any(self.anchors[:, 2:] <= 0):
            raise UnsupportedModel("Invalid detector anchors or scales")
        self.labels = task.get("labels", [])
        if self.labels and len(self.labels) != self.classes:
            raise UnsupportedModel("Label count does not match detector classes")

    def _boxes(self, raw, anchors):
        values = raw / self.scales
        cy = values[:, 0] * anchors[:, 3] + anchors[:, 1]
        cx = values[:, 1] * anchors[:, 2] + anchors[:, 0]
        if self.task["exponential_size"]:
            with np.errstate(over="raise", invalid="raise"):
                try:
                    sizes = np.exp(values[:, 2:])
                except FloatingPointError as exc:
                    raise ValueError("Nonfinite decoded box dimensions") from exc
        else:
            sizes = values[:, 2:]
        height, width = sizes[:, 0] * anchors[:, 3], sizes[:, 1] * anchors[:, 2]
        return np.stack((cx - width / 2, cy - height / 2, cx + width / 2, cy + height / 2), axis=1), height, width

    def decode(self, outputs, *, score_threshold=.5, iou_threshold=.5, max_results=20, class_aware=False):
        if not 0 <= score_threshold <= 1 or not 0 <= iou_threshold <= 1 or type(max_results) is not int \
                or not 1 <= max_results <= 1000:
            raise ValueError("Invalid confidence, IoU or result limit")
        raw = np.asarray(outputs[self.task["boxes_output"]])
        scores = np.asarray(outputs[self.task["scores_output"]])
        if raw.shape != (1, self.count, 4) or scores.shape != (1, self.count, self.classes):
            raise ValueError("Detector outputs do not match metadata")
        if not np.all(np.isfinite(raw)) or not np.all(np.isfinite(scores)):
            raise ValueError("Nonfinite detector output")
        raw, scores = raw[0], scores[0]
        classes = np.argmax(scores, axis=1)
        confidence = scores[np.arange(self.count), classes]
        if self.task["sigmoid_scores"]:
            confidence = 1 / (1 + np.exp(-np.clip(confidence, -80, 80)))
        selected = np.flatnonzero(confidence >= score_threshold)
        if not selected.size:
            return []
        boxes, height, width = self._boxes(raw[selected], self.anchors[selected])
        valid = np.flatnonzero((height > 0) & (width > 0) & np.all(np.isfinite(boxes), axis=1))
        order = valid[np.argsort(-confidence[selected[valid]], kind="stable")]
        areas = width * height
        keep = []
        while len(order) and len(keep) < max_results:
            best, rest = int(order[0]), order[1:]
            keep.append(best)
            lower = np.maximum(boxes[best, :2], boxes[rest, :2])
            upper = np.minimum(boxes[best, 2:], boxes[rest, 2:])
            inter = np.prod(np.maximum(upper - lower, 0), axis=1)
            union = areas[best] + areas[rest] - inter
            iou = np.divide(inter, union, out=np.zeros_like(inter), where=union > 0)
            drop = iou > iou_threshold
            if class_aware:
                drop &= classes[selected[rest]] == classes[selected[best]]
            order = rest[~drop]
        result = []
        for i in keep:
            source = selected[i]
            category = int(classes[source])
            box = np.clip(boxes[i], 0, 1)
            if box[2] <= box[0] or box[3] <= box[1]:
                continue
            label = self.labels[category] if self.labels else str(category)
            result.append(Detection(category, label, float(confidence[source]), tuple(float(v) for v in box)))
        return result


def _device_input(session, pixels, table):
    """Install `table` on the session's GPU (once per distinct table) and pass the pixels on."""
    if session.input_table is None or session.input_table is not table and not np.array_equal(session.input_table, table):
        session.set_input_table(table)
    return pixels


def _timings(t0, t1, t2, t3):
    return {"preprocess_ms": (t1 - t0) / 1e6, "inference_and_transfer_ms": (t2 - t1) / 1e6,
            "postprocess_ms": (t3 - t2) / 1e6, "total_ms": (t3 - t0) / 1e6}


class ObjectDetector:
    """Bundle-driven detector: preprocessing and anchors from the metadata, network on the GPU,
    box decoding on the host (top-k for the one-to-one YOLO head, NMS for fixed-anchor SSD)."""

    def __init__(self, model, *, library=None, pipeline="rpc", on_device=True):
        model = resolve(model)
        task = model.metadata.get("task", {})
        self.profile = task.get("preprocessing")
        self.on_device = bool(on_device)
        self.device_decode = False
        if task.get("kind") == "yolo_one_to_one":
            from .modern import YOLODecoder
            self.decoder = YOLODecoder(task, model.metadata.get("outputs", []), model.metadata["input"]["shape"])
        else:
            self.decoder = SSDDecoder(task)
        self.session = Session(model, library=library, pipeline=pipeline)
        if self.on_device and task.get("kind") == "yolo_one_to_one":
            self.session.set_yolo_decode(self.decoder.device_config())
            self.device_decode = True
        self.last_timings = {}

    def _prepare(self, image, options):
        spec = self.session.metadata["input"]
        if self.profile:
            from .modern import prepare_profile, profile_pixels
            if self.on_device:
                pixels, table, geometry = profile_pixels(image, spec, self.profile)
                x = _device_input(self.session, pixels, table)
            else:
                x, geometry = prepare_profile(image, spec, self.profile)
            return x, dict(options, geometry=geometry)
        if self.on_device:
            pixels, table, _ = image_pixels(image, spec, self.decoder.task["normalization"])
            return _device_input(self.session, pixels, table), options
        x, _ = prepare_image(image, spec, self.decoder.task["normalization"])
        return x, options

    def _limit(self, options):
        """Records to request from the GPU decoder: the validated max_results."""
        return self.decoder.check_options(**{k: v for k, v in options.items() if k != "geometry"})

    def detect(self, image, **options):
        t0 = time.perf_counter_ns()
        x, options = self._prepare(image, options)
        t1 = time.perf_counter_ns()
        if self.device_decode:
            records = self.session.detect_batch(x, self._limit(options))[0]
            t2 = time.perf_counter_ns()
            result = self.decoder.finish(records, **options)
        else:
            outputs = self.session.run(x)
            t2 = time.perf_counter_ns()
            result = self.decoder.decode(outputs, **options)
        self.last_timings = _timings(t0, t1, t2, time.perf_counter_ns())
        return result

    def detect_batch(self, images, **options):
        """Detections for each image of `images`, one GPU call for the whole batch."""
        t0 = time.perf_counter_ns()
        prepared = [self._prepare(image, options) for image in images]
        t1 = time.perf_counter_ns()
        x = np.concatenate([x for x, _ in prepared])
        if self.device_decode:
            records = self.session.detect_batch(x, self._limit(prepared[0][1]) if prepared else 1)
            t2 = time.perf_counter_ns()
            result = [self.decoder.finish(rec, **opts) for rec, (_, opts) in zip(records, prepared)]
        else:
            outputs = self.session.run_batch(x)
            t2 = time.perf_counter_ns()
            result = [self.decoder.decode(out, **opts) for out, (_, opts) in zip(outputs, prepared)]
        self.last_timings = _timings(t0, t1, t2, time.perf_counter_ns())
        return result

    def close(self):
        self.session.close()

    def __enter__(self):
        return self

    def __exit__(self, *args):
        self.close()


class ImageClassifier:
    """Classifier with bundled preprocessing, or explicit mean/std when the bundle has none."""

    def __init__(self, model, *, mean=None, std=None, labels=(), library=None, pipeline="rpc", on_device=True):
        model = resolve(model)
        task = model.metadata.get("task", {})
        self.profile = task.get("preprocessing") if task.get("kind") == "image_classification" else None
        if self.profile:
            if mean is not None or std is not None:
                raise ValueError("Bundled preprocessing is explicit; do not override normalization")
            if not labels:
                labels = task.get("labels", ())
        elif mean is None or std is None:
            raise ValueError("Provide mean/std or a bundle with classification preprocessing")
        self.softmax = bool(task.get("apply_softmax", False))
        outputs = model.metadata.get("outputs", [model.metadata["output"]])
        shape = outputs[0]["shape"]
        if len(outputs) != 1 or len(shape) < 2 or shape[0] != 1 or int(np.prod(shape)) != shape[-1]:
            raise UnsupportedModel("Classifier requires one class-vector output")
        if labels and len(labels) != shape[-1]:
            raise ValueError("Label count does not match model output")
        self.labels = list(labels)
        self.normalization = {"mean": mean, "std": std}
        self.output_spec = outputs[0]
        self.on_device = bool(on_device)
        self.session = Session(model, library=library, pipeline=pipeline)
        self.last_timings = {}

    def _prepare(self, image):
        spec = self.session.metadata["input"]
        if self.profile:
            from .modern import prepare_profile, profile_pixels
            if self.on_device:
                pixels, table, _ = profile_pixels(image, spec, self.profile)
                return _device_input(self.session, pixels, table)
            return prepare_profile(image, spec, self.profile)[0]
        if self.on_device:
            pixels, table, _ = image_pixels(image, spec, self.normalization)
            return _device_input(self.session, pixels, table)
        return prepare_image(image, spec, self.normalization)[0]

    def _top(self, raw, top_k):
        if self.output_spec.get("dequantize"):
            scores = raw
        else:
            q = self.output_spec["quantization"]
            scores = (raw.astype("f4") - q["zero_point"]) * q["scale"]
        if self.softmax:
            scores = np.exp(scores - scores.max())
            scores /= scores.sum()
        return [{"class_id": int(i), "label": self.labels[i] if self.labels else str(i), "score": float(scores[i])}
                for i in np.argsort(-scores, kind="stable")[:top_k]]

    def classify(self, image, *, top_k=5):
        if type(top_k) is not int or top_k < 1:
            raise ValueError("top_k must be positive")
        t0 = time.perf_counter_ns()
        x = self._prepare(image)
        t1 = time.perf_counter_ns()
        raw = self.session.run(x).reshape(-1)
        t2 = time.perf_counter_ns()
        result = self._top(raw, top_k)
        self.last_timings = _timings(t0, t1, t2, time.perf_counter_ns())
        return result

    def classify_batch(self, images, *, top_k=5):
        """Top-k classes for each image of `images`, one GPU call for the whole batch."""
        if type(top_k) is not int or top_k < 1:
            raise ValueError("top_k must be positive")
        t0 = time.perf_counter_ns()
        x = np.concatenate([self._prepare(image) for image in images])
        t1 = time.perf_counter_ns()
        raw = np.asarray(self.session.run_batch(x)).reshape(len(x), -1)
        t2 = time.perf_counter_ns()
        result = [self._top(row, top_k) for row in raw]
        self.last_timings = _timings(t0, t1, t2, time.perf_counter_ns())
        return result

    def close(self):
        self.session.close()

    def __enter__(self):
        return self

    def __exit__(self, *args):
        self.close()
