"""CPU: the oracle (C restatement) against the reference's own outputs.

tests/golden/*.npz were produced by the reference runtime compiled from its sources
(tests/golden/make_golden.py). Where that build is present (oracle/_ref), the oracle is also
compared to it live on fresh seeded inputs.
"""
import hashlib

import numpy as np
import pytest

import opcases
from conftest import model_path


@pytest.mark.parametrize("name", [n for n, _ in opcases.all_cases(1)])
def test_oracle_matches_reference_golden(name, oracle, golden_ops):
    plan = golden_ops[f"{name}/plan"].tobytes()
    x = golden_ops[f"{name}/x"]
    y = oracle.run(plan, x)
    np.testing.assert_array_equal(y, golden_ops[f"{name}/y"])


def test_golden_plans_are_regenerated_identically(golden_ops):
    for name, build in opcases.all_cases(1):
        plan, x = build(np.random.default_rng(7))
        assert plan == golden_ops[f"{name}/plan"].tobytes(), name
        np.testing.assert_array_equal(np.ascontiguousarray(x).reshape(-1).view(np.int8), golden_ops[f"{name}/x"])


@pytest.mark.parametrize("name,shape", [("mobilenetv4-small", (1, 224, 224, 3)), ("yolo26n-320", (1, 320, 320, 3))])
def test_oracle_matches_reference_on_bundled_models(name, shape, oracle, golden_models):
    from unoq_dsp.bundle import load
    model = load(model_path(name))
    assert hashlib.sha256(model.plan).digest() == golden_models[f"{name}/sha256"].tobytes()
    x = np.random.default_rng(0).integers(-128, 128, size=shape, dtype=np.int64).astype(np.int8)
    np.testing.assert_array_equal(oracle.run(model.plan, x), golden_models[f"{name}/y0"])


def test_scale_contract(oracle):
    """qnn.c:61-83 on hand-checked values: left shift, rounding, ties away from zero."""
    m = 1 << 30  # 0.5 in Q31
    assert oracle.scale(3, m, 0) == 2      # 1.5 rounds up (doubling high mul adds 2^30)
    assert oracle.scale(-3, m, 0) == -1    # -1.5 -> floor(-1.5 + 0.5) = -1
    assert oracle.scale(6, m, -1) == 2     # 3 / 2 = 1.5 -> ties away -> 2
    assert oracle.scale(-6, m, -1) == -2   # -3 / 2 -> ties away from zero -> -2
    assert oracle.scale(5, m, -1) == 2     # h = 3 (2.5 rounds up), then 3 / 2 ties away -> 2
    assert oracle.scale(1, m, 2) == 2      # (1 << 2) * 0.5


def test_live_reference_agrees_on_fresh_seeds(oracle):
    from oracle.oracle import REF_LIB, Reference
    if not REF_LIB.is_file():
        pytest.skip("reference build absent (oracle/_ref is built where the reference is mounted)")
    ref = Reference()
    for name, build in opcases.all_cases(1):
        for seed in (11, 12):
            plan, x = build(np.random.default_rng(seed))
            np.testing.assert_array_equal(oracle.run(plan, x), ref.run(plan, x), err_msg=name)
