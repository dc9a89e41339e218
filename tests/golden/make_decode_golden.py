"""Golden vectors for the host-side image and box paths, produced by the REFERENCE package.

Run where the reference checkout is mounted (it imports the reference's src/unoq_dsp in a
separate interpreter so it does not clash with this repository's package):

    UNOQ_REFERENCE_DIR=<reference checkout> python tests/golden/make_decode_golden.py

Writes decode.json: for seeded inputs, the reference's profile_lookup / image_lookup tables
(as SHA-256 of the bytes), prepare_profile / prepare_image outputs (SHA-256), the one-to-one YOLO
decode of the bundled detector's metadata on seeded raw int8 heads, and SSD fixed-anchor decodes
of a seeded synthetic task. tests/test_vision.py regenerates the same inputs and compares.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

OUT = Path(__file__).resolve().parent / "decode.json"
# the reference checkout: UNOQ_REFERENCE_DIR, else a `reference` directory beside this repository
REF_SRC = Path(os.environ.get("UNOQ_REFERENCE_DIR", Path(__file__).resolve().parents[3] / "reference")) / "src"

WORKER = r'''
import base64, hashlib, json, sys
import numpy as np
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[2])
from unoq_dsp.modern import YOLODecoder, prepare_profile, profile_lookup
from unoq_dsp.vision import SSDDecoder, prepare_image, image_lookup
import decode_cases as dc

def h(a): return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
def det(d): return [[x.class_id, x.label, x.score, list(x.box)] for x in d]
out = {"profile_lookup": [], "image_lookup": [], "prepare_profile": [], "prepare_image": [], "yolo": [], "ssd": []}
for args in dc.PROFILE_TABLES:
    out["profile_lookup"].append(h(profile_lookup(*args)))
for args in dc.IMAGE_TABLES:
    out["image_lookup"].append(h(image_lookup(*args)))
for case in dc.profile_cases():
    x, geometry = prepare_profile(case["image"], case["spec"], case["profile"])
    out["prepare_profile"].append([h(x), geometry])
for case in dc.image_cases():
    x, size = prepare_image(case["image"], case["spec"], case["normalization"])
    out["prepare_image"].append([h(x), list(size)])
task, outputs, shape = dc.yolo_contract()
decoder = YOLODecoder(task, outputs, shape)
for raw, geometry, options in dc.yolo_cases(outputs):
    out["yolo"].append(det(decoder.decode(raw, geometry=geometry, **options)))
for task, raw, options in dc.ssd_cases():
    out["ssd"].append(det(SSDDecoder(task).decode(raw, **options)))

# Whole pipelines on the bundled models: the reference's ImageClassifier / ObjectDetector with its
# Session replaced by the reference runtime built from source (oracle/_ref/libug_ref.so).
import ctypes as C
from unittest.mock import patch
from unoq_dsp import ImageClassifier, ObjectDetector, load
ref = C.CDLL(sys.argv[3])
ref.ug_load.argtypes = [C.c_void_p, C.c_uint32]
ref.ug_run.argtypes = [C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32]
ref.ug_output_bytes.restype = C.c_uint32

class RuntimeSession:
    def __init__(self, model, **kw):
        self.metadata = model.metadata
        self.plan = C.create_string_buffer(model.plan, len(model.plan))
        assert ref.ug_load(self.plan, len(model.plan)) == 0
    def run(self, x):
        x = np.ascontiguousarray(x)
        y = np.empty(ref.ug_output_bytes(), np.int8)
        assert ref.ug_run(x.ctypes.data, x.nbytes, y.ctypes.data, y.nbytes) == 0
        if not self.metadata.get("outputs"):
            return y.reshape(self.metadata["output"]["shape"])
        wire = y.view("u1"); res = {}
        for spec in self.metadata["outputs"]:
            res[spec["name"]] = wire[spec["packed_offset"]:spec["packed_offset"] + spec["bytes"]].view(spec["dtype"]).reshape(spec["shape"])
        return res
    def close(self): pass

out["classify"] = []; out["detect"] = []
with patch("unoq_dsp.vision.Session", RuntimeSession):
    clf = ImageClassifier(load(sys.argv[4] + "/mobilenetv4-small.uqmodel"))
    for image in dc.pipeline_images(224):
        out["classify"].append([[r["class_id"], r["label"], r["score"]] for r in clf.classify(image, top_k=5)])
    detector = ObjectDetector(load(sys.argv[4] + "/yolo26n-320.uqmodel"))
    for image in dc.pipeline_images(320):
        out["detect"].append(det(detector.detect(image, score_threshold=0.0, max_results=30)))
print(json.dumps(out))
'''


def main():
    here = Path(__file__).resolve().parent
    root = here.parents[1]
    res = subprocess.run([sys.executable, "-c", WORKER, str(REF_SRC), str(here),
                          str(root / "oracle" / "_ref" / "libug_ref.so"), str(root / "models")],
                         capture_output=True, text=True)
    if res.returncode:
        raise SystemExit(res.stderr)
    OUT.write_text(json.dumps(json.loads(res.stdout), indent=1) + "\n")
    print("wrote", OUT)


if __name__ == "__main__":
    main()
