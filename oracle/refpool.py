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


def _time_worker(args):
    """Seconds per image of the reference runtime on `plan` (one process, one core): one warm-up
    image, then `reps` timed images."""
    import time
    plan, ni, reps, seed = args
    for p in (str(ROOT), str(ROOT / "unoq-dsp_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from oracle.oracle import Reference
    ref = Reference()
    if ref.load(plan):
        raise RuntimeError("reference ug_load failed")
    x = np.random.default_rng(seed).integers(-128, 128, size=ni, dtype=np.int8)
    ref.run(plan, x)
    t0 = time.perf_counter()
    for _ in range(reps):
        ref.run(plan, x)
    return (time.perf_counter() - t0) / reps


def reference_timings(jobs, procs=None):
    """The reference C runtime (oracle/_ref/libug_ref.so, single-threaded off Hexagon) timed two
    ways per job (name, plan, input bytes, reps): on one core (one process alone) and on every
    core (`procs` processes at once, each running whole images). Returns {name: {...}}."""
    procs = max(1, procs or os.cpu_count() or 1)
    out = {}
    with mp.get_context("spawn").Pool(procs) as pool:
        for name, plan, ni, reps in jobs:
            one = pool.apply(_time_worker, ((bytes(plan), ni, reps, 1),))
            # every process times its own images after its load and warm-up; the slowest sets the rate
            per = pool.map(_time_worker, [(bytes(plan), ni, reps, 2 + i) for i in range(procs)], chunksize=1)
            out[name] = {"one_core_ms": round(one * 1e3, 3), "one_core_images_per_s": round(1.0 / one, 3),
                         "all_cores_images_per_s": round(procs / max(per), 3), "cores": procs,
                         "images_per_process": reps}
    return out
