"""The SURVEY §8 parity configurations as seeded one-layer plans (generators of BASELINE configs
0 and 1), from the package's synthetic-plan module (unoq_dsp.synth.baseline_config_cases), so the
tests and bench.py build the very same plans."""
import numpy as np

from unoq_dsp import synth

CONFIG1_SHAPES = synth.CONFIG1_SHAPES


def config_cases():
    return synth.baseline_config_cases()


def build(name, seed=11):
    """(plan bytes, input shape, output shape) of configuration `name`, from its seed."""
    return synth.baseline_config(name, seed)


def image(shape, seed):
    return np.random.default_rng(seed).integers(-128, 128, size=shape, dtype=np.int64).astype(np.int8)
