"""TEST INFRASTRUCTURE ONLY: the reference runtime over many images at once.

oracle/_ref/libug_ref.so (the reference's graph.c/qnn.c/gemm.c built for the host) runs one image
per call on one core, about 0.16 s for MobileNetV4 and 0.4 s for YOLO26n. To check hundreds of
images of a GPU batch, each worker of a `spawn` pool (never `fork`: a process forked after the
first CUDA call can hang) loads the plan once and runs whole images. Falls back to the C
restatement (oracle/liboracle.so, pinned to the reference by the golden fixtures) where the
reference build is absent. Used by tests/ and by bench.py's output check (after its timed
region), never by the product.
"""
import multiprocessing as mp
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
_STATE = {}


def _init(plan):
    for p in (str(ROOT), str(ROOT / "unoq-dsp_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from oracle.oracle import REF_LIB, Oracle, Reference
    if REF_LIB.is_file():
        ref = Reference()
        if ref.load(plan):
            raise RuntimeError("reference ug_load failed")
        _STATE.update(run=lambda x: ref.run(plan, x), kind="reference")
    else:
        orc = Oracle()
        _STATE.update(run=lambda x: orc.run(plan, x), kind="oracle")


def _one(x):
    return _STATE["run"](np.frombuffer(x, dtype=np.int8)).tobytes()


def checker_kind():
    from oracle.oracle import REF_LIB
    return "reference" if REF_LIB.is_file() else "oracle"


def reference_outputs(plan, images, procs=None):
    """Outputs of the reference runtime for `images` (a list of one-image int8 arrays), in order,
    as a (len(images), output_bytes) int8 array."""
    images = [np.ascontiguousarray(x).reshape(-1).view(np.int8).tobytes() for x in images]
    if not images:
        return np.empty((0, 0), dtype=np.int8)
    procs = max(1, min(procs or os.cpu_count() or 1, len(images)))
    with mp.get_context("spawn").Pool(procs, initializer=_init, initargs=(bytes(plan),)) as pool:
        outs = pool.map(_one, images, chunksize=max(1, len(images) // (4 * procs)))
    return np.stack([np.frombuffer(o, dtype=np.int8) for o in outs])
