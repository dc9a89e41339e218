"""The .uqmodel container: a fixed header, a JSON manifest and a UGN1 plan.

Container layout (little endian; the reference writes and reads the same bytes,
src/unoq_dsp/bundle.py:18-19, 66-81, so files move between the two unchanged):

    offset  size  field
         0     8  magic "UQMODEL\\0"
         8     4  container version (1)
        12     4  manifest bytes M (1 .. 4 MiB)
        16     4  plan bytes P (32 .. 17 MiB)
        20    32  SHA-256 of manifest || plan
        52     M  manifest: JSON object (input / output specs, packed output views, task, ...)
      52+M     P  plan: UGN1 header, tensor and op records, arena (runtime/graph.h:15-38)

``load`` accepts exactly the files the reference loader accepts and raises ``InvalidBundle``
for every file it rejects. The checks are written here as tables of named rules: the header
fields, the plan's header and tensor records, and the manifest's I/O, quantisation and packed
output sections.
"""
from dataclasses import dataclass
import hashlib
import json
import math
from pathlib import Path
import struct

import numpy as np

from .errors import InvalidBundle
from .limits import ARENA_BYTES, MAX_OPERATORS, MAX_PLAN_BYTES, MAX_TENSORS

MAGIC = b"UQMODEL\0"
CONTAINER_VERSION = 1
HEADER = struct.Struct("<8sIII32s")
MAX_MANIFEST = 4 * 1024 * 1024
PLAN_MAGIC = 0x55474E31
PLAN_HEADER = struct.Struct("<8I")
TENSOR_RECORD = struct.Struct("<12I")
OP_RECORD_BYTES = 32
# plan element types (runtime/graph.h:20): code -> numpy dtype
ELEMENT_TYPES = {1: np.dtype("<f4"), 2: np.dtype("u1"), 3: np.dtype("i1"), 4: np.dtype("<i4")}
BYTE_TYPES = (np.dtype("i1"), np.dtype("u1"))
MAX_PACKED_OUTPUTS = 32
# manifest keys a saved bundle keeps (the portable contract; development state is dropped)
PORTABLE_KEYS = ("input", "output", "arena_bytes", "plan_bytes", "macs", "dsp_threads", "source_sha256",
                 "source_format", "compiler_version", "memory_plan", "outputs", "task")
# exceptions a malformed manifest raises while it is read; each becomes InvalidBundle
_MANIFEST_FAULTS = (KeyError, TypeError, ValueError, OverflowError, RecursionError)


def _require(rules):
    """Raise InvalidBundle with the message of the first rule (message, failed) that fails; the
    rules are evaluated in order and stop at the first failure."""
    for message, failed in rules:
        if failed():
            raise InvalidBundle(message)


# ----------------------------------------------------------------------------------- plan

@dataclass(frozen=True)
class _TensorRecord:
    index: int
    offset: int
    size: int
    type: int
    rank: int
    dims: tuple
    constant: int
    reserved: tuple

    @classmethod
    def read(cls, plan, index):
        f = TENSOR_RECORD.unpack_from(plan, PLAN_HEADER.size + TENSOR_RECORD.size * index)
        return cls(index, f[0], f[1], f[2], f[3], tuple(f[4:8]), f[8], tuple(f[9:12]))

    @property
    def shape(self):
        return self.dims[:self.rank]


def _tensor_rules(t, version, arena, end):
    """Each descriptor: known element type, rank <= 4, positive dimensions, a 0/1 constant flag,
    zero reserved words, 128-byte aligned offsets that (before version 3) never step back, the
    bytes inside the arena and equal to shape x element size."""
    dtype = ELEMENT_TYPES.get(t.type)
    return [
        ("element type", lambda: dtype is None),
        ("rank", lambda: t.rank > 4),
        ("dimension", lambda: any(d <= 0 for d in t.shape)),
        ("constant flag", lambda: t.constant > 1),
        ("reserved words", lambda: any(t.reserved)),
        ("offset alignment", lambda: t.offset % 128 != 0),
        ("offset order", lambda: version < 3 and t.offset < end),
        ("arena bounds", lambda: t.offset + t.size > arena),
        ("byte count", lambda: math.prod(t.shape) * dtype.itemsize != t.size),
    ]


def plan_specs(plan):
    """Input and output descriptors of a UGN1 plan after the structural checks a bundle needs
    (the native loader validates the ops themselves)."""
    if not PLAN_HEADER.size <= len(plan) <= MAX_PLAN_BYTES:
        raise InvalidBundle("plan length out of range")
    magic, version, nt, no, arena, inp, out, threads = PLAN_HEADER.unpack_from(plan)
    _require([
        ("plan magic", lambda: magic != PLAN_MAGIC),
        ("plan version", lambda: version not in (2, 3)),
        ("tensor count", lambda: not 1 <= nt <= MAX_TENSORS),
        ("op count", lambda: not 1 <= no <= MAX_OPERATORS),
        ("arena size", lambda: not 0 < arena <= ARENA_BYTES),
        ("input / output index", lambda: max(inp, out) >= nt),
        ("thread field", lambda: threads > 1),
        ("plan length", lambda: len(plan) != PLAN_HEADER.size + TENSOR_RECORD.size * nt + OP_RECORD_BYTES * no + arena),
    ])
    io = {}
    end = 0
    for index in range(nt):
        t = _TensorRecord.read(plan, index)
        for reason, failed in _tensor_rules(t, version, arena, end):
            if failed():
                raise InvalidBundle(f"tensor {index}: bad {reason}")
        end = t.offset + t.size
        for role, wanted in (("input", inp), ("output", out)):
            if index == wanted:
                if t.constant:
                    raise InvalidBundle(f"the {role} tensor is a constant")
                io[role] = {"shape": t.shape, "dtype": ELEMENT_TYPES[t.type], "bytes": t.size}
    io.update(arena_bytes=arena, plan_bytes=len(plan), dsp_threads=1 + threads)
    return io


# ----------------------------------------------------------------------------------- manifest

def _quantization_ok(q, dtype):
    """Positive finite scale, integer zero point inside the element type's range."""
    bounds = np.iinfo(dtype)
    return (math.isfinite(q["scale"]) and q["scale"] > 0 and type(q["zero_point"]) is int
            and bounds.min <= q["zero_point"] <= bounds.max)


def _check_io(metadata, planned):
    """The manifest's input and output must describe the plan's; they take the plan's figures."""
    for role in ("input", "output"):
        spec, truth = metadata[role], planned[role]
        if tuple(spec["shape"]) != truth["shape"] or np.dtype(spec["dtype"]) != truth["dtype"]:
            raise InvalidBundle(f"manifest {role} differs from the plan")
        if "quantization" in spec and not _quantization_ok(spec["quantization"], truth["dtype"]):
            raise InvalidBundle(f"manifest {role} quantization")
        spec.update(truth)
    for key in ("arena_bytes", "plan_bytes", "dsp_threads"):
        metadata[key] = planned[key]


def _view_rules(view, seen, offset):
    shape = view["shape"]
    return [
        ("name", lambda: not isinstance(view["name"], str) or view["name"] in seen),
        ("rank", lambda: len(shape) > 4),
        ("dimensions", lambda: any(type(d) is not int or d <= 0 for d in shape)),
        ("element type", lambda: np.dtype(view["dtype"]) not in BYTE_TYPES),
        ("byte count", lambda: math.prod(shape) != view["bytes"]),
        ("packed offset", lambda: view["packed_offset"] != offset),
    ]


def _check_packed_outputs(metadata, planned):
    """Optional `outputs`: up to 32 named byte views laid end to end over the plan's (byte typed)
    output tensor, each with an optional dequantisation."""
    views = metadata["outputs"]
    if (not isinstance(views, list) or not 1 <= len(views) <= MAX_PACKED_OUTPUTS
            or planned["output"]["dtype"] not in BYTE_TYPES):
        raise InvalidBundle("packed outputs section")
    offset, seen = 0, set()
    for view in views:
        for reason, failed in _view_rules(view, seen, offset):
            if failed():
                raise InvalidBundle(f"packed output view: bad {reason}")
        seen.add(view["name"])
        offset += view["bytes"]
        view["shape"] = tuple(view["shape"])
        view["dtype"] = np.dtype(view["dtype"])
        if (view.get("dequantize") or "quantization" in view) and \
                not _quantization_ok(view["quantization"], view["dtype"]):
            raise InvalidBundle("packed output view: bad dequantization")
    if offset != planned["output"]["bytes"]:
        raise InvalidBundle("packed output views do not cover the plan's output")


def _read_manifest(text, plan):
    metadata = json.loads(text)
    if not isinstance(metadata, dict):
        raise InvalidBundle("the manifest is not a JSON object")
    planned = plan_specs(plan)
    _check_io(metadata, planned)
    if "outputs" in metadata:
        _check_packed_outputs(metadata, planned)
    return metadata


# ----------------------------------------------------------------------------------- files

def _json_value(value):
    if isinstance(value, np.dtype):
        return value.str
    if isinstance(value, np.generic):
        return value.item()
    raise TypeError(type(value).__name__)


@dataclass(frozen=True)
class CompiledModel:
    plan: bytes
    metadata: dict

    def save(self, path):
        planned = plan_specs(self.plan)
        for role in ("input", "output"):
            spec = self.metadata[role]
            if tuple(spec["shape"]) != planned[role]["shape"] or np.dtype(spec["dtype"]) != planned[role]["dtype"]:
                raise InvalidBundle(f"metadata {role} differs from the plan")
        kept = {key: self.metadata[key] for key in PORTABLE_KEYS if key in self.metadata}
        manifest = json.dumps(kept, default=_json_value, allow_nan=False, sort_keys=True,
                              separators=(",", ":")).encode()
        if len(manifest) > MAX_MANIFEST:
            raise InvalidBundle("manifest larger than 4 MiB")
        header = HEADER.pack(MAGIC, CONTAINER_VERSION, len(manifest), len(self.plan),
                             hashlib.sha256(manifest + self.plan).digest())
        Path(path).write_bytes(header + manifest + self.plan)


def load(path):
    """Read a .uqmodel file, verify its header, checksum, plan records and manifest."""
    with Path(path).open("rb") as f:
        raw = f.read(HEADER.size)
        if len(raw) != HEADER.size:
            raise InvalidBundle("file shorter than the container header")
        magic, version, n_manifest, n_plan, digest = HEADER.unpack(raw)
        _require([
            ("not a .uqmodel file", lambda: magic != MAGIC),
            ("unsupported container version", lambda: version != CONTAINER_VERSION),
            ("manifest length out of range", lambda: not 1 <= n_manifest <= MAX_MANIFEST),
            ("plan length out of range", lambda: not 32 <= n_plan <= MAX_PLAN_BYTES),
        ])
        body = f.read(n_manifest + n_plan + 1)  # one byte more than announced reveals trailing data
    if len(body) != n_manifest + n_plan:
        raise InvalidBundle("payload length differs from the header")
    if hashlib.sha256(body).digest() != digest:
        raise InvalidBundle("checksum mismatch")
    plan = body[n_manifest:]
    try:
        metadata = _read_manifest(body[:n_manifest], plan)
    except InvalidBundle:
        raise
    except _MANIFEST_FAULTS as exc:
        raise InvalidBundle(f"malformed manifest: {exc}") from exc
    return CompiledModel(plan, metadata)
