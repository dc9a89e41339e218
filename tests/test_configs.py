"""Parity on the two seeded configurations the reference's correctness claim is quoted on: config 0
(one pointwise INT8 conv, 1x56x56x64 -> 128) and config 1 (the depthwise 3x3/5x5, stride 1/2 sweep
over four shapes), at batch 1 and batch 256 (tests/configcases.py builds them).

tests/golden/configs.npz pins each plan and the reference runtime's output (SHA-256) for input
seeds 0 and 1; the oracle is checked against it on CPU, the CUDA path on the GPU, and at batch 256
the CUDA path is compared with the oracle image by image. Bit-exact throughout."""
import ctypes as C
import hashlib

import numpy as np
import pytest

import configcases
from conftest import GOLDEN
from gpuhelp import NativeSession

NAMES = [n for n, _ in configcases.config_cases()]


@pytest.fixture(scope="module")
def golden_configs():
    return np.load(GOLDEN / "configs.npz")


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).digest()


def test_config_plans_are_regenerated_identically(golden_configs):
    for name in NAMES:
        plan, _, _ = configcases.build(name)
        assert hashlib.sha256(plan).digest() == golden_configs[f"{name}/plan_sha256"].tobytes(), name


@pytest.mark.parametrize("name", NAMES)
def test_oracle_matches_reference_on_configs(name, oracle, golden_configs):
    plan, xs, _ = configcases.build(name)
    for seed in (0, 1):
        y = oracle.run(plan, configcases.image(xs, seed))
        assert sha(y) == golden_configs[f"{name}/y{seed}_sha256"].tobytes(), (name, seed)


@pytest.mark.gpu
@pytest.mark.parametrize("name", NAMES)
def test_config_batch1_matches_reference(name, native, golden_configs):
    """ug_load + ug_run, one image per call, against the reference's output digests."""
    plan, xs, zs = configcases.build(name)
    buf = C.create_string_buffer(plan, len(plan))
    assert native.ug_load(buf, len(plan)) == 0, native.ug_last_error()
    no = native.ug_output_bytes()
    assert no == int(np.prod(zs))
    for seed in (0, 1):
        x = configcases.image(xs, seed)
        y = np.empty(no, dtype=np.int8)
        assert native.ug_run(x.ctypes.data, x.nbytes, y.ctypes.data, no) == 0, native.ug_last_error()
        assert sha(y) == golden_configs[f"{name}/y{seed}_sha256"].tobytes(), (name, seed)


@pytest.mark.gpu
@pytest.mark.parametrize("name", NAMES)
def test_config_batch256_matches_oracle(name, native, oracle, golden_configs):
    """ug_infer_batch at 256 images (the batched config) against the oracle, image for image; the
    first two images are the golden seeds, so the batch also lands on the reference's digests."""
    plan, xs, _ = configcases.build(name)
    images = 256
    x = np.stack([configcases.image(xs, s) for s in range(images)])
    with NativeSession(native, plan) as s:
        got = s.run(x, images).reshape(images, -1)
    expect = oracle.run(plan, x, images).reshape(images, -1)
    bad = np.nonzero((got != expect).any(axis=1))[0]
    assert bad.size == 0, f"{name}: {bad.size} of {images} images differ (first {bad[:8].tolist()})"
    for seed in (0, 1):
        assert sha(got[seed]) == golden_configs[f"{name}/y{seed}_sha256"].tobytes(), (name, seed)
