"""The .uqmodel container: fixed header, JSON manifest, UGN1 plan.

Format (the reference's src/unoq_dsp/bundle.py:18-19, 66-81): a little-endian ``<8sIII32s``
header -- magic ``UQMODEL\\0``, version 1, manifest length, plan length, SHA-256 of
manifest+plan -- followed by the manifest and the plan. ``load`` applies the same checks as the
reference loader and raises ``InvalidBundle`` for the same conditions.
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
HEADER = struct.Struct("<8sIII32s")
MAX_MANIFEST = 4 * 1024 * 1024
_DTYPES = {1: np.dtype("<f4"), 2: np.dtype("u1"), 3: np.dtype("i1"), 4: np.dtype("<i4")}
_KEPT = ("input", "output", "arena_bytes", "plan_bytes", "macs", "dsp_threads", "source_sha256", "source_format",
         "compiler_version", "memory_plan", "outputs", "task")


def plan_specs(plan):
    """Input/output descriptors of a UGN1 plan after structural checks."""
    if not 32 <= len(plan) <= MAX_PLAN_BYTES:
        raise InvalidBundle("Invalid plan length")
    magic, version, nt, no, arena, inp, out, flags = struct.unpack_from("<8I", plan)
    if (magic != 0x55474E31 or version not in (2, 3) or not 1 <= nt <= MAX_TENSORS or not 1 <= no <= MAX_OPERATORS
            or not 0 < arena <= ARENA_BYTES or max(inp, out) >= nt or flags > 1
            or len(plan) != 32 + 48 * nt + 32 * no + arena):
        raise InvalidBundle("Unsupported or malformed plan header")
    specs = {}
    end = 0
    for i in range(nt):
        offset, size, typ, rank, d0, d1, d2, d3, constant, r0, r1, r2 = struct.unpack_from("<12I", plan, 32 + 48 * i)
        shape = (d0, d1, d2, d3)[:rank]
        bad = (typ not in _DTYPES or rank > 4 or any(d <= 0 for d in shape) or constant > 1 or (r0 or r1 or r2)
               or offset % 128 or (version < 3 and offset < end) or offset + size > arena
               or (typ in _DTYPES and math.prod(shape) * _DTYPES[typ].itemsize != size))
        if bad:
            raise InvalidBundle(f"Invalid tensor descriptor {i}")
        end = offset + size
        for name, index in (("input", inp), ("output", out)):
            if i == index:
                if constant:
                    raise InvalidBundle(f"{name} cannot be constant")
                specs[name] = {"shape": shape, "dtype": _DTYPES[typ], "bytes": size}
    specs.update(arena_bytes=arena, plan_bytes=len(plan), dsp_threads=1 + flags)
    return specs


def _json_default(value):
    if isinstance(value, np.dtype):
        return value.str
    if isinstance(value, np.generic):
        return value.item()
    raise TypeError(type(value).__name__)


def _check_quant(q, dtype, message):
    info = np.iinfo(dtype)
    if (not math.isfinite(q["scale"]) or q["scale"] <= 0 or type(q["zero_point"]) is not int
            or not info.min <= q["zero_point"] <= info.max):
        raise InvalidBundle(message)


@dataclass(frozen=True)
class CompiledModel:
    plan: bytes
    metadata: dict

    def save(self, path):
        checked = plan_specs(self.plan)
        for key in ("input", "output"):
            spec = self.metadata[key]
            if tuple(spec["shape"]) != checked[key]["shape"] or np.dtype(spec["dtype"]) != checked[key]["dtype"]:
                raise InvalidBundle("Metadata and plan disagree")
        manifest = json.dumps({k: self.metadata[k] for k in _KEPT if k in self.metadata}, default=_json_default,
                              allow_nan=False, sort_keys=True, separators=(",", ":")).encode()
        if len(manifest) > MAX_MANIFEST:
            raise InvalidBundle("Manifest too large")
        digest = hashlib.sha256(manifest + self.plan).digest()
        Path(path).write_bytes(HEADER.pack(MAGIC, 1, len(manifest), len(self.plan), digest) + manifest + self.plan)


def load(path):
    """Read and verify a .uqmodel bundle."""
    with Path(path).open("rb") as f:
        head = f.read(HEADER.size)
        if len(head) != HEADER.size:
            raise InvalidBundle("Truncated model header")
        magic, version, n_manifest, n_plan, digest = HEADER.unpack(head)
        if magic != MAGIC or version != 1 or not 1 <= n_manifest <= MAX_MANIFEST or not 32 <= n_plan <= MAX_PLAN_BYTES:
            raise InvalidBundle("Unsupported model format or length")
        payload = f.read(n_manifest + n_plan + 1)
    if len(payload) != n_manifest + n_plan or hashlib.sha256(payload).digest() != digest:
        raise InvalidBundle("Model length/checksum mismatch")
    try:
        metadata = json.loads(payload[:n_manifest])
        if not isinstance(metadata, dict):
            raise InvalidBundle("Expected a model manifest")
        plan = payload[n_manifest:]
        checked = plan_specs(plan)
        for name in ("input", "output"):
            spec = metadata[name]
            canon = checked[name]
            if tuple(spec["shape"]) != canon["shape"] or np.dtype(spec["dtype"]) != canon["dtype"]:
                raise InvalidBundle("Manifest I/O does not match the plan")
            if "quantization" in spec:
                _check_quant(spec["quantization"], canon["dtype"], "Invalid I/O quantization")
            spec.update(canon)
        for key in ("arena_bytes", "plan_bytes", "dsp_threads"):
            metadata[key] = checked[key]
        if "outputs" in metadata:
            outputs = metadata["outputs"]
            if (not isinstance(outputs, list) or not 1 <= len(outputs) <= 32
                    or checked["output"]["dtype"] not in (np.dtype("i1"), np.dtype("u1"))):
                raise InvalidBundle("Invalid multiple-output manifest")
            offset, names = 0, set()
            for spec in outputs:
                shape = spec["shape"]
                if (not isinstance(spec["name"], str) or spec["name"] in names or len(shape) > 4
                        or any(type(d) is not int or d <= 0 for d in shape)
                        or np.dtype(spec["dtype"]) not in (np.dtype("i1"), np.dtype("u1"))
                        or math.prod(shape) != spec["bytes"] or spec["packed_offset"] != offset):
                    raise InvalidBundle("Invalid packed output view")
                names.add(spec["name"])
                offset += spec["bytes"]
                spec["shape"] = tuple(shape)
                spec["dtype"] = np.dtype(spec["dtype"])
                if spec.get("dequantize") or "quantization" in spec:
                    _check_quant(spec["quantization"], spec["dtype"], "Invalid output dequantization")
            if offset != checked["output"]["bytes"]:
                raise InvalidBundle("Packed output length does not match plan")
    except (KeyError, TypeError, ValueError, OverflowError, RecursionError) as exc:
        if isinstance(exc, InvalidBundle):
            raise
        raise InvalidBundle(f"Invalid manifest: {exc}") from exc
    return CompiledModel(plan, metadata)
