"""Bundle-driven preprocessing and the one-to-one YOLO box decoder (host side).

Follows the reference's src/unoq_dsp/modern.py:
* ``profile_lookup`` (modern.py:10-18): the per-channel byte -> quantised input table.
* ``prepare_profile`` (modern.py:21-55): center-crop or letterbox resize, then the table.
* ``YOLODecoder`` (modern.py:58-103): distance-to-grid boxes, sigmoid scores, two-stage top-k.

The arithmetic is float32 in the same operation order as the reference, so the tables, boxes and
scores are identical to the reference's for identical int8 outputs. Image resizing and the final
per-detection geometry run on the host; the byte table and the top-k decode can run on the GPU
(``profile_pixels`` + ``Session.set_input_table``, ``YOLODecoder.device_config`` + ``finish``),
fed with the same float32 tables the host decoder computes, so both paths give identical results.
"""
from functools import lru_cache

import numpy as np

from .errors import UnsupportedModel


@lru_cache(maxsize=32)
def profile_lookup(mean, std, scale, zero, dtype):
    """256x3 table: byte b of channel c -> clip(rint(((b/255 - mean[c]) / std[c]) / scale) + zero).

    Float32 throughout, ties to even (np.rint), as the exporting pipeline does (modern.py:10-18).
    """
    byte = np.arange(256, dtype="f4")[:, None] / np.float32(255)
    normalised = (byte - np.asarray(mean, dtype="f4")) / np.asarray(std, dtype="f4")
    quantised = np.rint(normalised / np.float32(scale)) + zero
    info = np.iinfo(dtype)
    table = np.clip(quantised, info.min, info.max).astype(dtype)
    table.flags.writeable = False
    return table


def _as_rgb_image(image):
    from PIL import Image
    if isinstance(image, np.ndarray):
        if image.dtype != np.uint8 or image.ndim != 3 or image.shape[2] != 3:
            raise ValueError("Expected H×W×3 uint8 RGB")
        image = Image.fromarray(image)
    if not isinstance(image, Image.Image):
        raise TypeError("Expected Pillow image or RGB array")
    return image if image.mode == "RGB" else image.convert("RGB")


def _center_crop(image, oh, ow, crop_pct):
    from PIL import Image
    if oh != ow or not 0 < crop_pct <= 1:
        raise UnsupportedModel("Invalid square center crop")
    width, height = image.size
    side = int(oh / crop_pct)
    # shorter side -> `side`, aspect preserved (integer truncation as in modern.py:37)
    size = (side, int(side * height / width)) if width < height else (int(side * width / height), side)
    resized = image.resize(size, Image.Resampling.BICUBIC)
    left, top = round((size[0] - ow) / 2), round((size[1] - oh) / 2)
    return np.asarray(resized.crop((left, top, left + ow, top + oh)), dtype="u1")


def _letterbox(image, oh, ow):
    try:
        import cv2
    except ImportError as exc:
        raise UnsupportedModel("Letterbox preprocessing requires the vision extra (OpenCV)") from exc
    width, height = image.size
    ratio = min(ow / width, oh / height)
    nw, nh = round(width * ratio), round(height * ratio)
    if not nw or not nh:
        raise ValueError("Image aspect ratio is too extreme for this letterbox size")
    left, top = round((ow - nw) / 2 - .1), round((oh - nh) / 2 - .1)
    canvas = np.full((oh, ow, 3), 114, "u1")
    canvas[top:top + nh, left:left + nw] = cv2.resize(np.asarray(image), (nw, nh), interpolation=cv2.INTER_LINEAR)
    return canvas, {"ratio": ratio, "left": left, "top": top, "width": width, "height": height}


def prepare_profile(image, spec, profile):
    """One image -> (1, H, W, 3) quantised input and the letterbox geometry (or None)."""
    pixels, table, geometry = profile_pixels(image, spec, profile)
    return table[pixels[0], np.arange(3)][None], geometry


def profile_pixels(image, spec, profile):
    """One image -> ((1, H, W, 3) uint8 resized pixels, (256, 3) byte table, geometry or None):
    ``prepare_profile`` before its table lookup, for a GPU that applies the table."""
    image = _as_rgb_image(image)
    width, height = image.size
    if not width or not height:
        raise ValueError("Image dimensions must be positive")
    shape = tuple(spec["shape"])
    if len(shape) != 4 or shape[0] != 1 or shape[3] != 3:
        raise UnsupportedModel("Expected batch-one NHWC RGB")
    oh, ow = shape[1:3]
    geometry = None
    if profile["resize"] == "center_crop":
        pixels = _center_crop(image, oh, ow, float(profile["crop_pct"]))
    elif profile["resize"] == "letterbox":
        pixels, geometry = _letterbox(image, oh, ow)
    else:
        raise UnsupportedModel("Unknown image resize profile")
    mean = np.asarray(profile["mean"], dtype="f4")
    std = np.asarray(profile["std"], dtype="f4")
    if mean.shape != (3,) or std.shape != (3,) or not np.all(np.isfinite(mean)) or not np.all(np.isfinite(std)) \
            or np.any(std <= 0):
        raise UnsupportedModel("Invalid RGB normalization")
    q = spec["quantization"]
    table = profile_lookup(tuple(float(v) for v in mean), tuple(float(v) for v in std), q["scale"], q["zero_point"],
                           np.dtype(spec["dtype"]).str)
    return pixels[None], table, geometry


class YOLODecoder:
    """Raw distance-to-grid boxes and class logits of a one-to-one head; top-k, no NMS."""

    def __init__(self, task, outputs, input_shape):
        if task.get("kind") != "yolo_one_to_one" or task.get("schema") != 1:
            raise UnsupportedModel("Invalid YOLO task contract")
        self.task = task
        self.labels = task.get("labels", [])
        self.classes = task.get("num_classes")
        if type(self.classes) is not int or not 1 <= self.classes <= 4096 or len(self.labels) != self.classes:
            raise UnsupportedModel("Invalid detector labels")
        self.strides = task.get("strides")
        self.names = task.get("output_order")
        if self.strides != [8, 16, 32] or not isinstance(self.names, list) or len(self.names) != 6 \
                or len(set(self.names)) != 6:
            raise UnsupportedModel("Invalid detector head configuration")
        self.height, self.width = input_shape[1:3]
        self.specs = {o["name"]: o for o in outputs}
        self.anchors = []
        for level, stride in enumerate(self.strides):
            if self.height % stride or self.width % stride:
                raise UnsupportedModel("Input must be divisible by detector strides")
            h, w = self.height // stride, self.width // stride
            for name, channels in zip(self.names[2 * level:2 * level + 2], (4, self.classes)):
                spec = self.specs.get(name)
                if spec is None or tuple(spec["shape"]) != (1, h, w, channels) or np.dtype(spec["dtype"]) != np.int8:
                    raise UnsupportedModel("Detector output shape/type mismatch")
            yy, xx = np.mgrid[:h, :w]
            self.anchors.append(np.stack((xx + .5, yy + .5), axis=-1).astype("f4"))

    def _dequantised(self, outputs, name):
        spec = self.specs[name]
        value = np.asarray(outputs[name])
        if value.shape != tuple(spec["shape"]) or value.dtype != np.int8:
            raise ValueError("Unexpected raw detector output")
        q = spec["quantization"]
        return (value[0].astype("f4") - q["zero_point"]) * q["scale"]

    @staticmethod
    def check_options(score_threshold=.25, max_results=20, iou_threshold=None):
        """The decode options' validation (modern.py:80-83); returns max_results."""
        if iou_threshold is not None:
            raise ValueError("The one-to-one YOLO head does not use NMS; omit iou_threshold")
        if not 0 <= score_threshold <= 1 or type(max_results) is not int or not 1 <= max_results <= 300:
            raise ValueError("Invalid confidence or result limit")
        return max_results

    def _tables(self, name):
        """Per-level float32 tables over the 256 int8 codes, by the host decoder's own expressions."""
        q = self.specs[name]["quantization"]
        return (np.arange(-128, 128, dtype=np.int8).astype("f4") - q["zero_point"]) * q["scale"]

    def device_config(self, candidates=300):
        """The decoder as a native.UgYoloDecode for Session.set_yolo_decode: tensor offsets in the
        packed output, distance and sigmoid-score tables computed exactly as ``decode`` computes
        them, and order codes of the scores (np.unique ranks) so the GPU compares integers."""
        from .native import YOLO_MAX_LEVELS, UgYoloDecode
        if len(self.strides) > YOLO_MAX_LEVELS:
            raise UnsupportedModel("Too many detector levels for the GPU decoder")
        config = UgYoloDecode(levels=len(self.strides), classes=self.classes, candidates=candidates)
        scores = []
        for level in range(len(self.strides)):
            logits = self._tables(self.names[2 * level + 1])
            scores.append(1 / (1 + np.exp(-np.clip(logits, -80, 80))))
        _, codes = np.unique(np.stack(scores), return_inverse=True)
        codes = codes.reshape(len(self.strides), 256)
        for level, stride in enumerate(self.strides):
            box, score = self.specs[self.names[2 * level]], self.specs[self.names[2 * level + 1]]
            if "packed_offset" not in box or "packed_offset" not in score:
                raise UnsupportedModel("GPU decoding needs packed detector outputs")
            lv = config.level[level]
            lv.box_offset, lv.score_offset = box["packed_offset"], score["packed_offset"]
            lv.height, lv.width = self.height // stride, self.width // stride
            lv.stride = stride
            lv.distance[:] = self._tables(self.names[2 * level]).tolist()
            lv.score[:] = scores[level].tolist()
            lv.rank[:] = codes[level].tolist()
        return config

    def finish(self, records, *, geometry, score_threshold=.25, max_results=20, iou_threshold=None):
        """Detections from the GPU decoder's records of one image: ``decode`` after its top-k."""
        from .native import NO_ANCHOR
        from .vision import Detection
        self.check_options(score_threshold, max_results, iou_threshold)
        detections = []
        for record in records[:max_results]:
            if record["anchor"] == NO_ANCHOR:
                break
            confidence = float(record["score"])
            if confidence < score_threshold:
                break
            category = int(record["class_id"])
            box = np.array(record["box"], dtype="f4")
            box[[0, 2]] = (box[[0, 2]] - geometry["left"]) / (geometry["ratio"] * geometry["width"])
            box[[1, 3]] = (box[[1, 3]] - geometry["top"]) / (geometry["ratio"] * geometry["height"])
            box = np.clip(box, 0, 1)
            if not np.all(np.isfinite(box)) or box[2] <= box[0] or box[3] <= box[1]:
                continue
            detections.append(Detection(category, self.labels[category], confidence, tuple(float(v) for v in box)))
        return detections

    def decode(self, outputs, *, geometry, score_threshold=.25, max_results=20, iou_threshold=None):
        from .vision import Detection
        self.check_options(score_threshold, max_results, iou_threshold)
        all_boxes, all_scores = [], []
        for level, stride in enumerate(self.strides):
            dist = self._dequantised(outputs, self.names[2 * level])
            logits = self._dequantised(outputs, self.names[2 * level + 1])
            grid = self.anchors[level]
            all_boxes.append(np.concatenate((grid - dist[:, :, :2], grid + dist[:, :, 2:]), axis=-1).reshape(-1, 4) * stride)
            all_scores.append(1 / (1 + np.exp(-np.clip(logits.reshape(-1, self.classes), -80, 80))))
        boxes, scores = np.concatenate(all_boxes), np.concatenate(all_scores)
        # two-stage top-k: best 300 anchors by their top class, then the best (anchor, class) pairs
        anchors = np.argsort(-scores.max(1), kind="stable")[:min(300, len(scores))]
        flat = scores[anchors].reshape(-1)
        detections = []
        for j in np.argsort(-flat, kind="stable")[:max_results]:
            confidence = float(flat[j])
            if confidence < score_threshold:
                break
            category = int(j % self.classes)
            box = boxes[anchors[j // self.classes]].copy()
            box[[0, 2]] = (box[[0, 2]] - geometry["left"]) / (geometry["ratio"] * geometry["width"])
            box[[1, 3]] = (box[[1, 3]] - geometry["top"]) / (geometry["ratio"] * geometry["height"])
            box = np.clip(box, 0, 1)
            if not np.all(np.isfinite(box)) or box[2] <= box[0] or box[3] <= box[1]:
                continue
            detections.append(Detection(category, self.labels[category], confidence, tuple(float(v) for v in box)))
        return detections
