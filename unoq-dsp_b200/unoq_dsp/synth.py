"""Synthesise UGN1 plans without TFLite: the compile-time arithmetic of the reference compiler.

The reference lowers TFLite graphs with ``tflite.lower`` (src/unoq_dsp/tflite.py:17-314). That
module needs the ``tflite`` package at import time, which is not available here, so the few
formulas a plan needs are restated in this file:

* Q31 multiplier/exponent of a real scale (src/unoq_dsp/quantization.py:7-17, tflite.py:157-162);
* the packed conv weight layout (tflite.py:152-155, runtime/gemm.h:9);
* the corrected bias ``bias - (xz + 128) * sum(w)`` (tflite.py:156);
* fused activation limits (tflite.py:61-66) and SAME padding (tflite.py:138-139);
* the residual-ADD parameter block (quantization.py:31-41) and MUL/BMM/MEAN blocks
  (tflite.py:212-273).

Used by the tests and by bench.py to build the single-layer workloads (BASELINE configs 0/1)
and per-opcode parity cases. Plans written here load in the reference runtime unchanged.
"""
import math
import struct

import numpy as np

MAGIC = 0x55474E31
TYPES = {"f4": 1, "u1": 2, "i1": 3, "i4": 4}


def multiplier(value):
    """(Q31 integer, exponent) with value ~= integer * 2**(exponent - 31)."""
    if not math.isfinite(value) or value < 0:
        raise ValueError("multiplier needs a finite non-negative value")
    mantissa, exponent = math.frexp(value)
    integer = int(math.floor(mantissa * 2.0**31 + 0.5))
    if integer == 2**31:
        integer //= 2
        exponent += 1
    if exponent < -31:
        integer, exponent = 0, 0
    return integer, exponent


def fixed_multiply(values, m, shift):
    """Vectorised TFLite rounding multiply for shift <= 0 (quantization.py:20-28)."""
    v = np.asarray(values, dtype=np.int64)
    high = (v * m + (1 << 30)) >> 31
    if shift == 0:
        return high
    n = -shift
    mask = (1 << n) - 1
    return (high >> n) + ((high & mask) > ((mask >> 1) + (high < 0))).astype(np.int64)


def activation_limits(act, scale, zero):
    """int8 clamp bounds of a fused activation ('none', 'relu', 'relu6')."""
    if act == "none":
        return -128, 127
    if act == "relu":
        return max(-128, zero), 127
    if act == "relu6":
        return max(-128, zero), min(127, int(math.floor(6.0 / scale + 0.5)) + zero)
    raise ValueError(act)


def same_padding(size, out, kernel, stride, dilation):
    total = max(0, (out - 1) * stride + (kernel - 1) * dilation + 1 - size)
    return total // 2, total - total // 2


def pack_conv_weights(w):
    """w[oc, kh, kw, ic] int8 -> (packed bytes, kp) in the reference's INT8 packed layout."""
    oc, kh, kw, ic = w.shape
    k = kh * kw * ic
    kp = (k + 7) & ~7
    ocp = (oc + 3) & ~3
    full = np.zeros((ocp, kp), dtype=np.int8)
    full[:oc, :k] = w.reshape(oc, k)
    # byte (j/4)*kp*4 + (t/8)*32 + (j%4)*8 + t%8
    packed = full.reshape(ocp // 4, 4, kp // 8, 8).transpose(0, 2, 1, 3).reshape(-1)
    return np.ascontiguousarray(packed), kp


class PlanWriter:
    """Accumulates tensors (128-byte aligned, non-overlapping) and ops; ``build`` emits a plan."""

    def __init__(self, threads=1):
        self.tensors = []
        self.ops = []
        self.arena = bytearray()
        self.threads = threads

    def tensor(self, shape, dtype="i1", values=None):
        shape = tuple(int(d) for d in shape)
        dt = np.dtype({"f4": "<f4", "u1": "u1", "i1": "i1", "i4": "<i4"}[dtype])
        size = int(np.prod(shape)) * dt.itemsize
        off = (len(self.arena) + 127) & ~127
        self.arena.extend(bytes(off - len(self.arena)))
        if values is None:
            self.arena.extend(bytes(size))
        else:
            data = np.asarray(values, dtype=dt).reshape(-1)
            if data.size * dt.itemsize != size:
                raise ValueError("tensor values do not match the shape")
            self.arena.extend(data.tobytes())
        self.tensors.append(dict(offset=off, bytes=size, type=TYPES[dtype], shape=shape, constant=values is not None))
        return len(self.tensors) - 1

    def op(self, code, a, b, out, p=(0, 0, 0, 0)):
        p = [int(v) & 0xFFFFFFFF for v in p] + [0] * (4 - len(p))
        self.ops.append((code, a, b, out, *p))

    def build(self, input_id, output_id, version=2):
        header = struct.pack("<8I", MAGIC, version, len(self.tensors), len(self.ops), len(self.arena), input_id,
                             output_id, int(self.threads == 2))
        desc = b"".join(
            struct.pack("<12I", t["offset"], t["bytes"], t["type"], len(t["shape"]),
                        *(list(t["shape"]) + [1] * (4 - len(t["shape"]))), int(t["constant"]), 0, 0, 0)
            for t in self.tensors)
        ops = b"".join(struct.pack("<8I", *o) for o in self.ops)
        return header + desc + ops + bytes(self.arena)


def conv2d(pw, x, x_shape, xq, weights, bias, wscales, yq, *, stride=(1, 1), dilation=(1, 1), padding="same",
           act="none", depthwise=False, post=None, scalar=False, out_shape=None):
    """Append a conv (code 14) or depthwise (code 15) op; returns (output tensor, output shape).

    weights: [oc, kh, kw, ic] for conv, [kh, kw, c] for depthwise; wscales per output channel.
    xq / yq: (scale, zero_point). padding: 'same', 'valid' or (top, left, bottom, right).
    post: optional 256-byte table fused after the clamp (plan op p[1]).
    """
    n, ih, iw, ic = x_shape
    xs, xz = xq
    ys, yz = yq
    if depthwise:
        kh, kw, oc = weights.shape
        k = kh * kw
    else:
        oc, kh, kw, wic = weights.shape
        assert wic == ic
        k = kh * kw * ic
    sh, sw = stride
    dh, dw = dilation
    if padding == "same":
        oh, ow = -(-ih // sh), -(-iw // sw)
        pt, pb = same_padding(ih, oh, kh, sh, dh)
        pl, pr = same_padding(iw, ow, kw, sw, dw)
    else:
        pt, pl, pb, pr = (0, 0, 0, 0) if padding == "valid" else padding
        oh = (ih + pt + pb - (kh - 1) * dh - 1) // sh + 1
        ow = (iw + pl + pr - (kw - 1) * dw - 1) // sw + 1
    if out_shape is not None:
        oh, ow = out_shape
    lo, hi = activation_limits(act, ys, yz)
    if depthwise:
        packed = weights.reshape(-1).astype(np.int8)
        sums = weights.reshape(k, oc).astype(np.int64).sum(axis=0)
        kp = (k + 7) & ~7
    else:
        packed, kp = pack_conv_weights(weights.astype(np.int8))
        sums = weights.reshape(oc, k).astype(np.int64).sum(axis=1)
    corrected = np.asarray(bias, dtype=np.int64) - (int(xz) + 128) * sums
    mult, shift = zip(*(multiplier(float(xs) * float(s) / float(ys)) for s in np.broadcast_to(wscales, (oc,))))
    q = [kh, kw, sh, sw, dh, dw, pt, pl, pb, pr, oh, ow, int(xz), int(yz), lo, hi, ic, oc, kp, int(scalar)]
    config = np.array(q + corrected.tolist() + list(mult) + list(shift), dtype=np.int64)
    if config.min() < -2**31 or config.max() >= 2**31:
        raise ValueError("parameter block exceeds int32")
    wi = pw.tensor((len(packed),), "i1", packed)
    qi = pw.tensor((len(config),), "i4", config)
    z = pw.tensor((n, oh, ow, oc), "i1")
    p1 = pw.tensor((256,), "u1", post) + 1 if post is not None else 0
    pw.op(15 if depthwise else 14, x, wi, z, (qi, p1, 0, 0))
    return z, (n, oh, ow, oc)


def pool2d(pw, x, x_shape, q_lohi, kernel, stride, padding="same", is_max=True, zero=0):
    n, ih, iw, c = x_shape
    kh, kw = kernel
    sh, sw = stride
    if padding == "same":
        oh, ow = -(-ih // sh), -(-iw // sw)
        pt, pb = same_padding(ih, oh, kh, sh, 1)
        pl, pr = same_padding(iw, ow, kw, sw, 1)
    else:
        pt = pl = pb = pr = 0
        oh, ow = (ih - kh) // sh + 1, (iw - kw) // sw + 1
    lo, hi = q_lohi
    q = [kh, kw, sh, sw, 1, 1, pt, pl, pb, pr, oh, ow, zero, zero, lo, hi, c, c, 8, int(is_max)]
    qi = pw.tensor((20,), "i4", q)
    z = pw.tensor((n, oh, ow, c), "i1")
    pw.op(16, x, x, z, (qi, 0, 0, 0))
    return z, (n, oh, ow, c)


def add_parameters(xs, xz, bs, bz, ys, yz, lo, hi):
    """Residual ADD block: output multiplier/shift/zero/limits + two int32 tables (520 words)."""
    twice = 2 * max(xs, bs)
    xm, xsh = multiplier(xs / twice)
    bm, bsh = multiplier(bs / twice)
    ym, ysh = multiplier(twice / ((1 << 20) * ys))
    if ysh > 0:
        raise ValueError("ADD output scale too small")
    dom = np.arange(-128, 128, dtype=np.int64)
    tx = fixed_multiply((dom - xz) * (1 << 20), xm, xsh)
    tb = fixed_multiply((dom - bz) * (1 << 20), bm, bsh)
    return np.concatenate(([ym, ysh, yz, lo, hi, 0, 0, 0], tx, tb)).astype(np.int32)


def random_quant_conv(rng, x_shape, oc, kernel, stride, *, xq=(0.02, -3), yq=(0.05, 5), act="relu", depthwise=False,
                      dilation=(1, 1), padding="same", bias_bits=12, wscale_range=(1e-3, 1e-2)):
    """Weights/bias/scales drawn as BASELINE config 0: uniform int8 weights in [-127, 127],
    per-channel scales log-uniform in wscale_range, bias uniform +-2**bias_bits."""
    kh, kw = kernel
    ic = x_shape[3]
    shape = (kh, kw, oc) if depthwise else (oc, kh, kw, ic)
    w = rng.integers(-127, 128, size=shape, dtype=np.int64).astype(np.int8)
    lo, hi = np.log(wscale_range[0]), np.log(wscale_range[1])
    ws = np.exp(rng.uniform(lo, hi, size=oc))
    bias = rng.integers(-(1 << bias_bits), (1 << bias_bits) + 1, size=oc)
    return dict(weights=w, bias=bias, wscales=ws, xq=xq, yq=yq, act=act, stride=stride, depthwise=depthwise,
                dilation=dilation, padding=padding)


def single_conv_plan(rng, x_shape, oc, kernel, stride, **kw):
    """A one-op conv/depthwise plan; returns (plan bytes, input shape, output shape)."""
    spec = random_quant_conv(rng, x_shape, oc, kernel, stride, **kw)
    pw = PlanWriter()
    x = pw.tensor(x_shape, "i1")
    z, zshape = conv2d(pw, x, x_shape, spec["xq"], spec["weights"], spec["bias"], spec["wscales"], spec["yq"],
                       stride=stride, dilation=spec["dilation"], padding=spec["padding"], act=spec["act"],
                       depthwise=spec["depthwise"])
    return pw.build(x, z), x_shape, zshape


# BASELINE configs 0 and 1 as seeded one-layer plans. Config 0: an INT8 pointwise conv on
# 1x56x56x64 -> 128 channels (input scale 0.02, zero point -3; per-channel weight scales
# log-uniform in [1e-3, 1e-2]; bias uniform +-2^12; output scale 0.05, zero point 5, ReLU clamp
# [5, 127]). Config 1: the depthwise sweep (3x3 and 5x5, stride 1 and 2, SAME) over 1x112x112x32,
# 1x56x56x96, 1x28x28x192 and 1x14x14x576 with the same quantisation generator.
CONFIG1_SHAPES = [(1, 112, 112, 32), (1, 56, 56, 96), (1, 28, 28, 192), (1, 14, 14, 576)]


def baseline_config_cases():
    """(name, builder) pairs; builder(rng) returns (plan bytes, input shape, output shape)."""
    cases = [("config0_pw", lambda r: single_conv_plan(r, (1, 56, 56, 64), 128, (1, 1), (1, 1)))]
    for shape in CONFIG1_SHAPES:
        for k in (3, 5):
            for s in (1, 2):
                name = f"config1_dw{k}_s{s}_{shape[1]}x{shape[3]}"
                cases.append((name, lambda r, shape=shape, k=k, s=s:
                              single_conv_plan(r, shape, shape[3], (k, k), (s, s), depthwise=True)))
    return cases


def baseline_config(name, seed=11):
    """(plan bytes, input shape, output shape) of configuration `name`, from its seed."""
    import numpy as np
    return dict(baseline_config_cases())[name](np.random.default_rng(seed))
