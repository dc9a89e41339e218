"""Malformed-plan variants for loader error-code parity (runtime/graph.c:50-216).

Each variant mutates one field of a small valid plan; the reference's ug_load code for each is
recorded in tests/golden/codes.npz and our loader must return the same number.
"""
import struct

import numpy as np

import opcases

H = struct.Struct("<8I")
T = struct.Struct("<12I")
O = struct.Struct("<8I")


def _base():
    plan, _ = opcases.block_case(np.random.default_rng(3), hw=4)
    return bytearray(plan)


def _fields(plan):
    magic, version, nt, no, arena, inp, out, flags = H.unpack_from(plan, 0)
    return nt, no


def _tensor_off(i):
    return 32 + 48 * i


def _op_off(plan, i):
    nt, _ = _fields(plan)
    return 32 + 48 * nt + 32 * i


def _set_u32(plan, off, value):
    struct.pack_into("<I", plan, off, value & 0xFFFFFFFF)


def variants():
    out = []
    base = _base()
    nt, no = _fields(base)
    out.append(("valid", bytes(base)))
    out.append(("truncated", bytes(base[:16])))
    p = bytearray(base); _set_u32(p, 0, 0x12345678); out.append(("bad magic", bytes(p)))
    p = bytearray(base); _set_u32(p, 4, 4); out.append(("bad version", bytes(p)))
    p = bytearray(base); _set_u32(p, 28, 2); out.append(("bad thread flag", bytes(p)))
    out.append(("length mismatch", bytes(base + b"\0" * 128)))
    p = bytearray(base); _set_u32(p, _tensor_off(1), T.unpack_from(base, _tensor_off(1))[0] + 4)
    out.append(("unaligned tensor", bytes(p)))
    p = bytearray(base); _set_u32(p, _tensor_off(1) + 8, 9); out.append(("bad tensor type", bytes(p)))
    p = bytearray(base); _set_u32(p, _tensor_off(0) + 32, 1); out.append(("constant input", bytes(p)))
    p = bytearray(base); _set_u32(p, _op_off(base, 0) + 4, nt + 5); out.append(("op input out of range", bytes(p)))
    p = bytearray(base); _set_u32(p, _op_off(base, 1) + 4, O.unpack_from(base, _op_off(base, 2))[3])
    out.append(("op reads undefined tensor", bytes(p)))
    p = bytearray(base); _set_u32(p, _op_off(base, 0), 99); out.append(("unknown opcode", bytes(p)))
    p = bytearray(base); _set_u32(p, _op_off(base, 0) + 24, 7); out.append(("conv stray p[2]", bytes(p)))
    # conv parameter block: change kernel height so the output size no longer matches
    qid = O.unpack_from(base, _op_off(base, 0))[4]
    qoff = 32 + 48 * nt + 32 * no + T.unpack_from(base, _tensor_off(qid))[0]
    p = bytearray(base); _set_u32(p, qoff, 3); out.append(("conv kh mismatch", bytes(p)))
    p = bytearray(base); _set_u32(p, qoff + 4 * 19, 5); out.append(("conv bad flags", bytes(p)))
    p = bytearray(base); _set_u32(p, qoff + 4 * 15, 200); out.append(("conv clamp out of range", bytes(p)))
    # add parameter block (op 3 is the residual ADD)
    aq = O.unpack_from(base, _op_off(base, 3))[4]
    aoff = 32 + 48 * nt + 32 * no + T.unpack_from(base, _tensor_off(aq))[0]
    p = bytearray(base); _set_u32(p, aoff + 4, 3); out.append(("add positive shift", bytes(p)))
    p = bytearray(base); _set_u32(p, 24, O.unpack_from(base, _op_off(base, 0))[4]); out.append(("output constant", bytes(p)))
    # version 3 with two live tensors sharing bytes
    p = bytearray(base); _set_u32(p, 4, 3)
    t1 = T.unpack_from(base, _tensor_off(O.unpack_from(base, _op_off(base, 0))[3]))
    t2i = O.unpack_from(base, _op_off(base, 1))[3]
    _set_u32(p, _tensor_off(t2i), t1[0])
    out.append(("v3 lifetime overlap", bytes(p)))
    p = bytearray(base); _set_u32(p, 4, 3); out.append(("valid v3", bytes(p)))
    return out
