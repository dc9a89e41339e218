"""The SURVEY §8 parity configurations as seeded one-layer plans (generators of BASELINE configs
0 and 1): config 0 is an INT8 pointwise conv on 1x56x56x64 -> 128 channels (input scale 0.02,
zero point -3; per-channel weight scales log-uniform in [1e-3, 1e-2]; bias uniform +-2^12; output
scale 0.05, zero point 5, ReLU clamp [5, 127]); config 1 is the depthwise sweep (3x3 and 5x5,
stride 1 and 2, SAME) over 1x112x112x32, 1x56x56x96, 1x28x28x192 and 1x14x14x576 with the same
quantisation generator."""
import numpy as np

from unoq_dsp import synth

CONFIG1_SHAPES = [(1, 112, 112, 32), (1, 56, 56, 96), (1, 28, 28, 192), (1, 14, 14, 576)]


def config_cases():
    cases = [("config0_pw", lambda r: synth.single_conv_plan(r, (1, 56, 56, 64), 128, (1, 1), (1, 1)))]
    for shape in CONFIG1_SHAPES:
        for k in (3, 5):
            for s in (1, 2):
                name = f"config1_dw{k}_s{s}_{shape[1]}x{shape[3]}"
                cases.append((name, lambda r, shape=shape, k=k, s=s:
                              synth.single_conv_plan(r, shape, shape[3], (k, k), (s, s), depthwise=True)))
    return cases


def build(name, seed=11):
    """(plan bytes, input shape, output shape) of configuration `name`, from its seed."""
    return dict(config_cases())[name](np.random.default_rng(seed))


def image(shape, seed):
    return np.random.default_rng(seed).integers(-128, 128, size=shape, dtype=np.int64).astype(np.int8)
