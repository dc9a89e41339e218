"""Generate the committed golden fixtures from the REFERENCE runtime itself.

Run where the reference checkout is mounted (it builds oracle/_ref/libug_ref.so from the
reference's own runtime/graph.c, qnn.c, gemm.c -- see oracle/Makefile):

    make -C oracle ref REF=<reference checkout> && python tests/golden/make_golden.py

The bundled models are read from models/ (staged by __graft_entry__.build()), else from the
checkout named by UNOQ_REFERENCE_DIR (default: a `reference` directory beside this repository).

Writes:
* ops.npz     -- every case of tests/opcases.py at scale 1: plan bytes, input, and the
                 reference's output (ug_load + ug_run of libug_ref.so).
* models.npz  -- for the two bundled models: the SHA-256 of the plan, seeded input images
                 (regenerated from the seed, not stored) and the reference's raw outputs.
* configs.npz -- the §8 parity configurations (tests/configcases.py): SHA-256 of each plan and
                 of the reference's output for input seeds 0 and 1 (tensors are regenerated).
* codes.npz   -- for each malformed-plan variant of tests/plancorrupt.py (regenerated at test
                 time, identified by SHA-256), the reference loader's error code.

The reference has no golden tensors of its own (its kernel tests compare against LiteRT's
interpreter, which is absent here); these fixtures pin our oracle to the reference instead.
"""
import hashlib
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path[:0] = [str(ROOT), str(ROOT / "unoq-dsp_b200"), str(ROOT / "tests")]

from oracle.oracle import Reference  # noqa: E402
import configcases  # noqa: E402
import opcases  # noqa: E402
import plancorrupt  # noqa: E402

OUT = Path(__file__).resolve().parent
MODELS = {"mobilenetv4-small": (1, 224, 224, 3), "yolo26n-320": (1, 320, 320, 3)}
MODEL_SEEDS = (0, 1)


def model_dir():
    local = ROOT / "models"
    if (local / "mobilenetv4-small.uqmodel").is_file():
        return local
    return Path(os.environ.get("UNOQ_REFERENCE_DIR", ROOT.parent / "reference")) / "models"


def main():
    ref = Reference()
    arrays = {}
    for name, build in opcases.all_cases(1):
        plan, x = build(np.random.default_rng(7))
        y = ref.run(plan, x)
        arrays[f"{name}/plan"] = np.frombuffer(plan, dtype=np.uint8)
        arrays[f"{name}/x"] = np.ascontiguousarray(x).reshape(-1).view(np.int8)
        arrays[f"{name}/y"] = y
    np.savez_compressed(OUT / "ops.npz", **arrays)

    carrays = {}
    for name, _ in configcases.config_cases():
        plan, xs, _ = configcases.build(name)
        carrays[f"{name}/plan_sha256"] = np.frombuffer(hashlib.sha256(plan).digest(), dtype=np.uint8)
        for seed in (0, 1):
            y = ref.run(plan, configcases.image(xs, seed))
            carrays[f"{name}/y{seed}_sha256"] = np.frombuffer(hashlib.sha256(y.tobytes()).digest(), dtype=np.uint8)
    np.savez_compressed(OUT / "configs.npz", **carrays)


    from unoq_dsp.bundle import load
    marrays = {}
    for name, shape in MODELS.items():
        model = load(model_dir() / f"{name}.uqmodel")
        marrays[f"{name}/sha256"] = np.frombuffer(hashlib.sha256(model.plan).digest(), dtype=np.uint8)
        for seed in MODEL_SEEDS:
            x = np.random.default_rng(seed).integers(-128, 128, size=shape, dtype=np.int64).astype(np.int8)
            marrays[f"{name}/y{seed}"] = ref.run(model.plan, x)
    np.savez_compressed(OUT / "models.npz", **marrays)

    carrays = {}
    for i, (label, plan) in enumerate(plancorrupt.variants()):
        carrays[f"{i}/sha256"] = np.frombuffer(hashlib.sha256(plan).digest(), dtype=np.uint8)
        carrays[f"{i}/code"] = np.array([ref.load(plan)], dtype=np.int32)
        carrays[f"{i}/label"] = np.frombuffer(label.encode(), dtype=np.uint8)
    np.savez_compressed(OUT / "codes.npz", **carrays)
    print("wrote", sorted(p.name for p in OUT.glob("*.npz")))


if __name__ == "__main__":
    main()
