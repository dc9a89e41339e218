"""Seeded one-op and few-op plans covering every INT8 opcode of the plan ABI.

Each builder returns (plan_bytes, input_array). Shapes are parameterised by `scale` so the same
case runs small (CPU oracle, golden fixtures) and large (GPU parity). Edge cases the reference
tests pin are included: ragged channel counts, stride/dilation/padding mixes, requantisation
with left shifts and negative ties, post-LUT fusion, saturating clamps, adj flags for BMM.
"""
import math

import numpy as np

from unoq_dsp import synth
from unoq_dsp.synth import PlanWriter, conv2d, multiplier


def _rand_input(rng, shape):
    return rng.integers(-128, 128, size=shape, dtype=np.int64).astype(np.int8)


def conv_case(rng, x_shape, oc, kernel, stride, **kw):
    plan, xs, _ = synth.single_conv_plan(rng, x_shape, oc, kernel, stride, **kw)
    return plan, _rand_input(rng, xs)


def conv_post_case(rng, x_shape, oc, kernel, stride, depthwise=False):
    """Conv/depthwise with a fused 256-entry post table (YOLO's SiLU-style fusion)."""
    spec = synth.random_quant_conv(rng, x_shape, oc, kernel, stride, depthwise=depthwise, act="none")
    pw = PlanWriter()
    x = pw.tensor(x_shape)
    table = rng.integers(0, 256, size=256).astype(np.uint8)
    z, _ = conv2d(pw, x, x_shape, spec["xq"], spec["weights"], spec["bias"], spec["wscales"], spec["yq"],
                  stride=stride, act="none", depthwise=depthwise, post=table)
    return pw.build(x, z), _rand_input(rng, x_shape)


def conv_shift_case(rng, x_shape, oc, kernel):
    """Output scale small enough that multipliers exceed one: positive exponents (pre-shift)."""
    spec = synth.random_quant_conv(rng, x_shape, oc, kernel, (1, 1), xq=(0.02, 1), yq=(2e-6, 0), act="none",
                                   bias_bits=4, wscale_range=(1e-3, 2e-3))
    w = spec["weights"]
    w[:] = np.clip(w // 32, -4, 4)
    pw = PlanWriter()
    x = pw.tensor(x_shape)
    z, _ = conv2d(pw, x, x_shape, spec["xq"], w, spec["bias"], spec["wscales"], spec["yq"], act="none")
    xin = rng.integers(-3, 4, size=x_shape).astype(np.int8)
    return pw.build(x, z), xin


def conv_ties_case(rng):
    """1x1 identity-like conv with exponents 1..15 below zero and small biases: exercises the
    ties-away-from-zero rounding on negative values (the reference pins this in
    tests/test_modern_ops.py:66-73)."""
    c = 16
    x_shape = (1, 4, 8, c)
    w = np.zeros((c, 1, 1, c), dtype=np.int8)
    for j in range(c):
        w[j, 0, 0, j] = 1 if j % 2 else -1
    pw = PlanWriter()
    x = pw.tensor(x_shape)
    ws = np.array([2.0 ** -(1 + j % 15) for j in range(c)])
    z, _ = conv2d(pw, x, x_shape, (1.0, 0), w, np.arange(-8, 8), ws, (1.0, 0), padding="valid", act="none")
    xin = np.resize(np.arange(-128, 128, dtype=np.int64), int(np.prod(x_shape))).astype(np.int8).reshape(x_shape)
    return pw.build(x, z), xin


def pool_case(rng, x_shape, kernel, stride, is_max, padding="same"):
    pw = PlanWriter()
    x = pw.tensor(x_shape)
    z, _ = synth.pool2d(pw, x, x_shape, (-100, 120), kernel, stride, padding=padding, is_max=is_max, zero=-3)
    return pw.build(x, z), _rand_input(rng, x_shape)


def add_case(rng, shape):
    pw = PlanWriter()
    x = pw.tensor(shape)
    b = pw.tensor(shape)
    # b must be an activation defined before the add: produce it from x by a LUT op.
    table = rng.integers(0, 256, size=256).astype(np.uint8)
    t = pw.tensor((256,), "u1", table)
    pw.op(22, x, t, b)
    q = synth.add_parameters(0.05, -3, 0.08, 7, 0.1, -1, -120, 127)
    qi = pw.tensor((520,), "i4", q)
    z = pw.tensor(shape)
    pw.op(18, x, b, z, (qi, 0, 0, 0))
    return pw.build(x, z), _rand_input(rng, shape)


def mul_case(rng, shape):
    pw = PlanWriter()
    x = pw.tensor(shape)
    t = pw.tensor((256,), "u1", rng.integers(0, 256, size=256).astype(np.uint8))
    b = pw.tensor(shape)
    pw.op(22, x, t, b)
    qm, qs = multiplier(0.05 * 0.04 / 0.03)
    qi = pw.tensor((7,), "i4", [-3, 5, 2, qm, qs, -128, 127])
    z = pw.tensor(shape)
    pw.op(25, x, b, z, (qi, 0, 0, 0))
    return pw.build(x, z), _rand_input(rng, shape)


def lut_case(rng, shape, out_dtype="i1"):
    pw = PlanWriter()
    x = pw.tensor(shape)
    t = pw.tensor((256,), "u1", rng.integers(0, 256, size=256).astype(np.uint8))
    z = pw.tensor(shape, out_dtype)
    pw.op(22, x, t, z)
    return pw.build(x, z), _rand_input(rng, shape)


def mean_parameters(count, xs, xz, ys, yz):
    """MEAN block as the reference compiler forms it (tflite.py:267-272)."""
    qm, qs = multiplier(xs / ys)
    adjust = min(count.bit_length() - 1, 32, 31 + qs)
    qm = (qm << adjust) // count
    qs -= adjust
    return [count, xz, yz, qm, qs]


def mean_case(rng, shape):
    n, h, w, c = shape
    pw = PlanWriter()
    x = pw.tensor(shape)
    qi = pw.tensor((5,), "i4", mean_parameters(h * w, 0.05, -7, 0.03, 4))
    z = pw.tensor((n, 1, 1, c))
    pw.op(24, x, qi, z)
    return pw.build(x, z), _rand_input(rng, shape)


def concat_case(rng, shape_a, shape_b, axis):
    pw = PlanWriter()
    x = pw.tensor(shape_a)
    # b: a slice of a LUT of x keeps it an activation of the right shape
    t = pw.tensor((256,), "u1", rng.integers(0, 256, size=256).astype(np.uint8))
    xa = pw.tensor(shape_a)
    pw.op(22, x, t, xa)
    b = pw.tensor(shape_b)
    pw.op(26, xa, xa, b, (0, 0, 0, 0))
    zshape = list(shape_a)
    zshape[axis] += shape_b[axis]
    z = pw.tensor(tuple(zshape))
    pw.op(20, x, b, z, (axis, 0, 0, 0))
    return pw.build(x, z), _rand_input(rng, shape_a)


def c2f_bytes_case(rng, hw, c):
    """YOLO's C2f byte ops: a tensor split in two by innermost-axis slices, each half through a
    table, then a chain of innermost-axis concats, concat(concat(concat(t0, t1), x), s1), where
    s1 also feeds its table (so that slice stays a copy)."""
    shape, half = (1, hw, hw, c), (1, hw, hw, c // 2)
    pw = PlanWriter()
    x = pw.tensor(shape)
    tables = [pw.tensor((256,), "u1", rng.integers(0, 256, size=256).astype(np.uint8)) for _ in range(2)]
    s0, s1 = pw.tensor(half), pw.tensor(half)
    pw.op(26, x, x, s0, (0, 0, 0, 0))
    pw.op(26, x, x, s1, (0, 0, 0, c // 2))
    t0, t1 = pw.tensor(half), pw.tensor(half)
    pw.op(22, s0, tables[0], t0)
    pw.op(22, s1, tables[1], t1)
    c1 = pw.tensor((1, hw, hw, c))
    pw.op(20, t0, t1, c1, (3, 0, 0, 0))
    c2 = pw.tensor((1, hw, hw, 2 * c))
    pw.op(20, c1, x, c2, (3, 0, 0, 0))
    z = pw.tensor((1, hw, hw, 2 * c + c // 2))
    pw.op(20, c2, s1, z, (3, 0, 0, 0))
    return pw.build(x, z), _rand_input(rng, shape)


def slice_case(rng, shape, begin, size):
    pw = PlanWriter()
    x = pw.tensor(shape)
    z = pw.tensor(size)
    pw.op(26, x, x, z, tuple(begin) + (0,) * (4 - len(begin)))
    return pw.build(x, z), _rand_input(rng, shape)


def transpose_case(rng, shape, perm):
    pw = PlanWriter()
    x = pw.tensor(shape)
    z = pw.tensor(tuple(shape[p] for p in perm))
    pw.op(10, x, x, z, tuple(perm) + (0,) * (4 - len(perm)))
    return pw.build(x, z), _rand_input(rng, shape)


def resize_case(rng, shape, out_hw):
    n, ih, iw, c = shape
    oh, ow = out_hw
    rows = (np.floor(np.arange(oh) * (ih / oh)).astype(np.int64) * iw * c)
    cols = (np.floor(np.arange(ow) * (iw / ow)).astype(np.int64) * c)
    pw = PlanWriter()
    x = pw.tensor(shape)
    b = pw.tensor((oh + ow,), "i4", np.concatenate((rows, cols)))
    z = pw.tensor((n, oh, ow, c))
    pw.op(21, x, b, z)
    return pw.build(x, z), _rand_input(rng, shape)


def pad_case(rng, shape, pads, value=-5):
    pads = np.asarray(pads, dtype=np.int64).reshape(4, 2)
    pw = PlanWriter()
    x = pw.tensor(shape)
    b = pw.tensor((8,), "i4", pads.reshape(-1))
    z = pw.tensor(tuple(np.asarray(shape) + pads.sum(axis=1)))
    pw.op(23, x, b, z, (value, 0, 0, 0))
    return pw.build(x, z), _rand_input(rng, shape)


def pack_case(rng, shape):
    """Three outputs packed: x itself, a LUT of x, a slice of x (op 19 list semantics)."""
    pw = PlanWriter()
    x = pw.tensor(shape)
    t = pw.tensor((256,), "u1", rng.integers(0, 256, size=256).astype(np.uint8))
    y1 = pw.tensor(shape)
    pw.op(22, x, t, y1)
    half = (shape[0], shape[1], shape[2], max(1, shape[3] // 2))
    y2 = pw.tensor(half)
    pw.op(26, x, x, y2, (0, 0, 0, 0))
    lst = pw.tensor((3,), "i4", [y1, x, y2])
    total = 2 * int(np.prod(shape)) + int(np.prod(half))
    z = pw.tensor((total,))
    pw.op(19, y1, lst, z)
    return pw.build(x, z), _rand_input(rng, shape)


def bmm_case(rng, batch, m, k, n, adj_x=0, adj_y=0):
    a_shape = (batch, k, m) if adj_x else (batch, m, k)
    b_shape = (batch, n, k) if adj_y else (batch, k, n)
    pw = PlanWriter()
    x = pw.tensor((int(np.prod(a_shape)) + int(np.prod(b_shape)),))
    a = pw.tensor(a_shape)
    pw.op(26, x, x, pw.tensor((int(np.prod(a_shape)),)), (0, 0, 0, 0))
    flat_a = len(pw.tensors) - 1
    pw.op(5, flat_a, flat_a, a)
    b = pw.tensor(b_shape)
    flat_b = pw.tensor((int(np.prod(b_shape)),))
    pw.op(26, x, x, flat_b, (int(np.prod(a_shape)), 0, 0, 0))
    pw.op(5, flat_b, flat_b, b)
    qm, qs = multiplier(0.02 * 0.03 / 0.5)
    qi = pw.tensor((7,), "i4", [-5, 3, 1, qm, qs, adj_x, adj_y])
    z = pw.tensor((batch, m, n))
    pw.op(27, a, b, z, (qi, 0, 0, 0))
    return pw.build(x, z), _rand_input(rng, (int(np.prod(a_shape)) + int(np.prod(b_shape)),))


def softmax_exact_case(rng, rows, width, scale=0.1):
    lut = [2147483647] + [int(round(2147483647 * math.exp(-i * scale))) for i in range(1, 256)]
    lut = np.minimum.accumulate(np.asarray(lut, dtype=np.int64))
    pw = PlanWriter()
    x = pw.tensor((1, rows, width))
    b = pw.tensor((257,), "i4", np.concatenate(([width], lut)))
    z = pw.tensor((1, rows, width))
    pw.op(28, x, b, z)
    return pw.build(x, z), _rand_input(rng, (1, rows, width))


def softmax_table_case(rng, rows, width, scale=0.05):
    table = [1 << 24] + [int(round((1 << 24) * math.exp(-i * scale))) for i in range(1, 256)]
    q = [1, 1, 1, 1, 1, 1, 0, 0, 0, 0, 1, 1, -128, -128, -128, 127, width, width, 8, 0] + table
    pw = PlanWriter()
    x = pw.tensor((1, rows, width))
    qi = pw.tensor((len(q),), "i4", q)
    z = pw.tensor((1, rows, width))
    pw.op(17, x, x, z, (qi, 0, 0, 0))
    return pw.build(x, z), _rand_input(rng, (1, rows, width))


def block_case(rng, hw=14, c=32, expand=96, conv_second=False):
    """Inverted-residual block: pw expand -> dw 3x3 -> pw project -> residual add (the projection
    is the add's first operand, or its second with conv_second)."""
    x_shape = (1, hw, hw, c)
    pw = PlanWriter()
    x = pw.tensor(x_shape)
    s1 = synth.random_quant_conv(rng, x_shape, expand, (1, 1), (1, 1), xq=(0.05, -3), yq=(0.04, -128))
    h, hs = conv2d(pw, x, x_shape, s1["xq"], s1["weights"], s1["bias"], s1["wscales"], s1["yq"], act="relu")
    s2 = synth.random_quant_conv(rng, hs, expand, (3, 3), (1, 1), xq=(0.04, -128), yq=(0.03, -128), depthwise=True)
    d, ds = conv2d(pw, h, hs, s2["xq"], s2["weights"], s2["bias"], s2["wscales"], s2["yq"], act="relu",
                   depthwise=True)
    s3 = synth.random_quant_conv(rng, ds, c, (1, 1), (1, 1), xq=(0.03, -128), yq=(0.06, 2), act="none")
    p, _ = conv2d(pw, d, ds, s3["xq"], s3["weights"], s3["bias"], s3["wscales"], s3["yq"], act="none")
    q = synth.add_parameters(0.06, 2, 0.05, -3, 0.07, 0, -128, 127)
    qi = pw.tensor((520,), "i4", q)
    z = pw.tensor(x_shape)
    pw.op(18, x if conv_second else p, p if conv_second else x, z, (qi, 0, 0, 0))
    return pw.build(x, z, version=2), _rand_input(rng, x_shape)


def all_cases(scale=1):
    """(name, builder) pairs; scale multiplies spatial sizes for the GPU runs."""
    s = scale
    return [
        ("conv_pw_c0", lambda r: conv_case(r, (1, 8 * s, 8 * s, 64), 128, (1, 1), (1, 1))),
        ("conv_pw_ragged", lambda r: conv_case(r, (1, 5 * s, 7, 48), 40, (1, 1), (1, 1), act="none")),
        # N tiles that are not powers of two: one 192-wide tile in four 48-column parts, three
        # 192-wide tiles, four 256-wide tiles whose last holds 192 channels, 80 channels in a
        # 96-wide tile, and a 3x3 conv with 96 channels on the 8-warp epilogue
        ("conv_pw_oc192", lambda r: conv_case(r, (1, 6 * s, 7, 96), 192, (1, 1), (1, 1))),
        ("conv_pw_oc576", lambda r: conv_case(r, (1, 3 * s, 7, 96), 576, (1, 1), (1, 1), act="none")),
        ("conv_pw_oc960", lambda r: conv_case(r, (1, 2 * s, 7, 128), 960, (1, 1), (1, 1))),
        ("conv_pw_oc80", lambda r: conv_case(r, (1, 5 * s, 9, 32), 80, (1, 1), (1, 1))),
        ("conv_3x3_oc96", lambda r: conv_case(r, (1, 6 * s, 9, 32), 96, (3, 3), (1, 1))),
        ("conv_3x3_s1", lambda r: conv_case(r, (1, 9 * s, 7, 16), 24, (3, 3), (1, 1))),
        ("conv_3x3_s2", lambda r: conv_case(r, (1, 10 * s, 10, 32), 16, (3, 3), (2, 2), xq=(0.03, 17))),
        ("conv_stem_rgb", lambda r: conv_case(r, (1, 16 * s, 12, 3), 16, (3, 3), (2, 2), xq=(0.02, -13))),
        ("conv_5x5_dil2_valid", lambda r: conv_case(r, (1, 12 * s, 11, 8), 4, (5, 5), (1, 1), dilation=(2, 2),
                                                    padding=(1, 0, 2, 3), act="relu6")),
        ("conv_rgb_band", lambda r: conv_case(r, (1, 10 * s, 16, 3), 16, (3, 3), (2, 2), xq=(0.02, 9))),
        # few input channels (the stems' row-GEMM path): padding on every side, stride 1, ic 1 and 4,
        # a post table, several column groups
        ("conv_rows_rgb_s2", lambda r: conv_case(r, (1, 9 * s, 32, 3), 32, (3, 3), (2, 2), xq=(0.02, -7))),
        ("conv_rows_rgb_s1", lambda r: conv_case(r, (1, 6 * s, 16, 3), 16, (3, 3), (1, 1), xq=(0.02, 4))),
        ("conv_rows_ic4_post", lambda r: conv_post_case(r, (1, 7 * s, 20, 4), 16, (3, 3), (2, 2))),
        ("conv_rows_ic1", lambda r: conv_case(r, (1, 5 * s, 48, 1), 32, (3, 3), (2, 2), act="relu6")),
        # 64-channel 3x3 inputs (row GEMM with three window blocks per kernel row)
        ("conv_rows_ic64_s1", lambda r: conv_case(r, (1, 7 * s, 12, 64), 16, (3, 3), (1, 1))),
        ("conv_rows_ic64_s2", lambda r: conv_case(r, (1, 9 * s, 14, 64), 64, (3, 3), (2, 2), xq=(0.03, -9))),
        # 33-64-channel inputs with at most 32 outputs at stride 2 (three or four window blocks per
        # kernel row), and 48 channels (three blocks) at strides 1 and 2
        ("conv_rows_ic64_s2_oc32", lambda r: conv_case(r, (1, 9 * s, 14, 64), 32, (3, 3), (2, 2), xq=(0.03, -9))),
        ("conv_rows_ic48_s2_oc16", lambda r: conv_case(r, (1, 9 * s, 15, 48), 16, (3, 3), (2, 2), xq=(0.02, 6))),
        ("conv_rows_ic48_s1_oc32", lambda r: conv_case(r, (1, 7 * s, 12, 48), 32, (3, 3), (1, 1))),
        # 48-column epilogue parts (G = 2 pixels x 96 channels)
        ("conv_rows_oc96_s2", lambda r: conv_case(r, (1, 9 * s, 16, 16), 96, (3, 3), (2, 2))),
        # 24 / 32-channel 3x3 inputs
        ("conv_rows2_ic32_s2", lambda r: conv_case(r, (1, 9 * s, 22, 32), 32, (3, 3), (2, 2), xq=(0.03, 11))),
        ("conv_rows2_ic32_s1", lambda r: conv_case(r, (1, 6 * s, 13, 32), 16, (3, 3), (1, 1))),
        ("conv_rows2_ic24_post", lambda r: conv_post_case(r, (1, 5 * s, 11, 24), 32, (3, 3), (1, 1))),
        # input channels a multiple of 32 (the per-tap TMA path): dilation, 32 / 64 / 128-byte
        # channel chunks, several N tiles, a 2 x 3 kernel with a post table
        ("conv_taps_ic64_dil2", lambda r: conv_case(r, (1, 9 * s, 11, 64), 32, (3, 3), (1, 1), dilation=(2, 2))),
        ("conv_taps_ic96_s2", lambda r: conv_case(r, (1, 11 * s, 9, 96), 48, (3, 3), (2, 2), xq=(0.03, -40))),
        ("conv_taps_ic128_oc320", lambda r: conv_case(r, (1, 5 * s, 6, 128), 320, (3, 3), (1, 1), act="none")),
        ("conv_taps_2x3_post", lambda r: conv_post_case(r, (1, 7 * s, 8, 32), 16, (2, 3), (1, 1))),
        ("conv_ic8_band", lambda r: conv_case(r, (1, 6 * s, 10, 8), 24, (3, 3), (1, 1))),
        # row GEMM with fewer than 16 output channels: a 16-column epilogue chunk spans 2 or 4
        # pixels, each with its own border correction
        ("conv_rows_oc8", lambda r: conv_case(r, (1, 9 * s, 11, 16), 8, (3, 3), (1, 1))),
        ("conv_rows_oc8_s2", lambda r: conv_case(r, (1, 10 * s, 13, 16), 8, (3, 3), (2, 2))),
        ("conv_rows_oc4_3x3", lambda r: conv_case(r, (1, 7 * s, 9, 8), 4, (3, 3), (1, 1))),
        ("conv_rows_oc4_1x1", lambda r: conv_case(r, (1, 6 * s, 10, 16), 4, (1, 1), (1, 1), act="none")),
        ("conv_rgb_odd_width", lambda r: conv_case(r, (1, 9 * s, 13, 3), 16, (3, 3), (2, 2), xq=(0.02, -5))),
        ("conv_ic8_small", lambda r: conv_case(r, (1, 9 * s, 11, 8), 16, (3, 3), (1, 1))),
        ("conv_ic16_small_post", lambda r: conv_post_case(r, (1, 8 * s, 10, 16), 8, (3, 3), (2, 2))),
        ("conv_fc", lambda r: conv_case(r, (1, 1, 1, 96), 40, (1, 1), (1, 1), act="none")),
        ("conv_wide_k", lambda r: conv_case(r, (1, 4 * s, 5, 256), 64, (3, 3), (1, 1))),
        ("conv_post_lut", lambda r: conv_post_case(r, (1, 6 * s, 6, 32), 32, (3, 3), (1, 1))),
        ("conv_shift_pos", lambda r: conv_shift_case(r, (1, 4 * s, 4, 16), 8, (1, 1))),
        ("conv_ties", lambda r: conv_ties_case(r)),
        ("dw3_s1", lambda r: conv_case(r, (1, 9 * s, 8, 32), 32, (3, 3), (1, 1), depthwise=True)),
        ("dw3_s2", lambda r: conv_case(r, (1, 11 * s, 9, 48), 48, (3, 3), (2, 2), depthwise=True)),
        ("dw5_s1", lambda r: conv_case(r, (1, 7 * s, 7, 64), 64, (5, 5), (1, 1), depthwise=True, act="none")),
        ("dw5_s2", lambda r: conv_case(r, (1, 14 * s, 14, 16), 16, (5, 5), (2, 2), depthwise=True)),
        ("dw3_c6", lambda r: conv_case(r, (1, 5 * s, 5, 6), 6, (3, 3), (1, 1), depthwise=True)),
        ("dw3_post_lut", lambda r: conv_post_case(r, (1, 6 * s, 6, 24), 24, (3, 3), (1, 1), depthwise=True)),
        ("dw3_s2_wide", lambda r: conv_case(r, (1, 13 * s, 19, 96), 96, (3, 3), (2, 2), depthwise=True)),
        ("dw5_s1_post", lambda r: conv_post_case(r, (1, 9 * s, 11, 32), 32, (5, 5), (1, 1), depthwise=True)),
        ("dw3_s1_c48_none", lambda r: conv_case(r, (1, 5 * s, 21, 48), 48, (3, 3), (1, 1), depthwise=True,
                                                act="none")),
        # tensor-core depthwise shapes: odd 5x5 stride 2 (four phase planes), two whole images per
        # tile (14x14 stride 2 -> 7x7), 128-channel slices over a 40-wide row (3 rows per tile)
        ("dw5_s2_c64", lambda r: conv_case(r, (1, 15 * s, 13, 64), 64, (5, 5), (2, 2), depthwise=True)),
        ("dw3_s2_c128_img2", lambda r: conv_case(r, (1, 14, 14, 128), 128, (3, 3), (2, 2), depthwise=True)),
        ("dw3_s1_c256_wide", lambda r: conv_case(r, (1, 3 * s, 40, 256), 256, (3, 3), (1, 1), depthwise=True,
                                                 act="none")),
        ("pool_max5", lambda r: pool_case(r, (1, 10 * s, 10, 16), (5, 5), (1, 1), True)),
        ("pool_avg3_s2", lambda r: pool_case(r, (1, 9 * s, 7, 8), (3, 3), (2, 2), False)),
        ("pool_avg2_valid", lambda r: pool_case(r, (1, 8 * s, 8, 4), (2, 2), (2, 2), False, padding="valid")),
        ("add", lambda r: add_case(r, (1, 7 * s, 5, 16))),
        ("mul", lambda r: mul_case(r, (1, 6 * s, 5, 8))),
        ("lut_i8", lambda r: lut_case(r, (1, 5 * s, 7, 9))),
        ("lut_u8", lambda r: lut_case(r, (1, 3 * s, 3, 16), out_dtype="u1")),
        ("mean", lambda r: mean_case(r, (1, 7, 7, 40 * s))),
        ("concat_c", lambda r: concat_case(r, (1, 4 * s, 5, 16), (1, 4 * s, 5, 8), 3)),
        ("c2f_bytes", lambda r: c2f_bytes_case(r, 5 * s, 32)),
        ("c2f_bytes_odd", lambda r: c2f_bytes_case(r, 3 * s, 24)),
        ("concat_h", lambda r: concat_case(r, (1, 4 * s, 5, 16), (1, 2, 5, 16), 1)),
        ("slice", lambda r: slice_case(r, (1, 6 * s, 7, 16), (0, 1, 2, 4), (1, 3, 4, 8))),
        ("transpose_nchw", lambda r: transpose_case(r, (1, 5 * s, 6, 12), (0, 3, 1, 2))),
        ("transpose_3d", lambda r: transpose_case(r, (2, 7 * s, 9), (0, 2, 1))),
        # rows and columns multiples of 4 (the word transpose): one matrix per block, and many
        # small matrices per block with a partial last chunk
        ("transpose_words", lambda r: transpose_case(r, (2, 10, 10, 64 * s), (0, 3, 1, 2))),
        ("transpose_words_many", lambda r: transpose_case(r, (13, 3, 12, 20 * s), (0, 1, 3, 2))),
        ("resize2x", lambda r: resize_case(r, (1, 5 * s, 6, 8), (10 * s, 12))),
        ("pad", lambda r: pad_case(r, (1, 4 * s, 5, 6), [0, 0, 1, 2, 2, 1, 0, 0])),
        ("pad_channels", lambda r: pad_case(r, (1, 3, 4 * s, 5), [0, 1, 0, 0, 1, 0, 2, 3])),
        ("pack", lambda r: pack_case(r, (1, 4 * s, 3, 6))),
        ("bmm", lambda r: bmm_case(r, 2, 10 * s, 16, 12)),
        ("bmm_adj", lambda r: bmm_case(r, 2, 9, 20, 7 * s, adj_x=1, adj_y=1)),
        # attention shapes (q^T k and v attn^T), K not a multiple of 4, one operand transposed
        ("bmm_attn_qk", lambda r: bmm_case(r, 2, 100, 32, 25 * s)),
        ("bmm_attn_v", lambda r: bmm_case(r, 2, 16 * s, 100, 100, adj_y=1)),
        ("bmm_odd_k", lambda r: bmm_case(r, 3, 7 * s, 13, 9, adj_x=1)),
        ("softmax_exact", lambda r: softmax_exact_case(r, 10 * s, 100)),
        ("softmax_table", lambda r: softmax_table_case(r, 6 * s, 33)),
        ("block", lambda r: block_case(r, hw=7 * s)),
        ("block_conv_second", lambda r: block_case(r, hw=5 * s, c=48, expand=64, conv_second=True)),
    ]
