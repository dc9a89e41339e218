"""Seeded .uqmodel files for the container loader's accept / reject behaviour: one valid bundle
(a small add plan with a manifest carrying quantisation, two packed output views and a task) and
mutations of every field the loader checks -- the container header, the checksum, the plan's
header and tensor records, the manifest's I/O specs, quantisation and packed output views.

`cases()` returns (label, file bytes). Both loaders read the same bytes: the reference's
(src/unoq_dsp/bundle.py, run by make_bundle_golden.py) and this repository's (tests/test_bundle.py).
The bytes are built here, not stored; bundle.json holds each case's SHA-256 and the reference's
verdict."""
import hashlib
import json
import struct

import numpy as np

HEADER = struct.Struct("<8sIII32s")
MAGIC = b"UQMODEL\0"


def _plan(version=2, threads=0, input_const=0, tensor_edits=None, header_edits=None, out_type=3, trailing=0):
    """A 3-tensor, 1-op UGN1 plan: int8 input (1, 4, 4, 8), int8 constant (520,) q-block-like
    words, int8 output (1, 4, 4, 8) (packed outputs view it as 8 + 120 bytes)."""
    arena = 128 * 4 + 2176
    tensors = [
        [0, 128, 3, 4, 1, 4, 4, 8, input_const, 0, 0, 0],
        [256, 2080, 4, 1, 520, 0, 0, 0, 1, 0, 0, 0],
        [2432, 128, out_type, 4, 1, 4, 4, 8, 0, 0, 0, 0],
    ]
    if out_type in (1, 4):  # a 4-byte element output of the same shape
        tensors[2] = [2432, 512, out_type, 4, 1, 4, 4, 8, 0, 0, 0, 0]
        arena = 2432 + 512
    for (i, field), value in (tensor_edits or {}).items():
        tensors[i][field] = value
    header = [0x55474E31, version, 3, 1, arena, 0, 2, threads]
    for field, value in (header_edits or {}).items():
        header[field] = value
    body = struct.pack("<8I", *header)
    for t in tensors:
        body += struct.pack("<12I", *[v & 0xFFFFFFFF for v in t])
    body += struct.pack("<8I", 18, 0, 0, 2, 1, 0, 0, 0)
    arena_bytes = np.random.default_rng(3).integers(0, 256, size=arena, dtype=np.int64).astype(np.uint8).tobytes()
    return body + arena_bytes + b"\0" * trailing


def _manifest(**edits):
    m = {
        "input": {"shape": [1, 4, 4, 8], "dtype": "|i1", "quantization": {"scale": 0.02, "zero_point": -3}},
        "output": {"shape": [1, 4, 4, 8], "dtype": "|i1", "quantization": {"scale": 0.05, "zero_point": 5}},
        "outputs": [
            {"name": "boxes", "shape": [2, 4], "dtype": "|i1", "bytes": 8, "packed_offset": 0,
             "dequantize": True, "quantization": {"scale": 0.1, "zero_point": 0}},
            {"name": "scores", "shape": [120], "dtype": "|u1", "bytes": 120, "packed_offset": 8},
        ],
        "task": {"kind": "detector", "labels": ["a", "b"]},
        "macs": 1024, "compiler_version": "test",
    }
    for path, value in edits.items():
        node, keys = m, path.split("/")
        for k in keys[:-1]:
            node = node[int(k)] if isinstance(node, list) else node[k]
        last = keys[-1]
        if value is _DELETE:
            del node[last]
        elif isinstance(node, list):
            node[int(last)] = value
        else:
            node[last] = value
    return m


_DELETE = object()


def _pack(manifest, plan, magic=MAGIC, version=1, n_manifest=None, n_plan=None, digest=None, tail=b"", text=None):
    raw = text if text is not None else json.dumps(manifest, sort_keys=True, separators=(",", ":")).encode()
    digest = digest if digest is not None else hashlib.sha256(raw + plan).digest()
    head = HEADER.pack(magic, version, len(raw) if n_manifest is None else n_manifest,
                       len(plan) if n_plan is None else n_plan, digest)
    return head + raw + plan + tail


def cases():
    good_plan, good = _plan(), _manifest()
    out = [("valid", _pack(good, good_plan))]
    add = lambda label, blob: out.append((label, blob))  # noqa: E731
    # container header and payload
    add("truncated header", _pack(good, good_plan)[:40])
    add("bad magic", _pack(good, good_plan, magic=b"UQMODEL1"))
    add("container version 2", _pack(good, good_plan, version=2))
    add("manifest length 0", _pack(good, good_plan, n_manifest=0))
    add("manifest length over 4 MiB", _pack(good, good_plan, n_manifest=4 * 1024 * 1024 + 1))
    add("plan length 31", _pack(good, good_plan, n_plan=31))
    add("plan length over 17 MiB", _pack(good, good_plan, n_plan=17 * 1024 * 1024 + 1))
    add("payload short", _pack(good, good_plan)[:-1])
    add("payload has a trailing byte", _pack(good, good_plan, tail=b"\0"))
    add("checksum wrong", _pack(good, good_plan, digest=b"\1" * 32))
    # manifest text and structure
    add("manifest not JSON", _pack(None, good_plan, text=b"{not json"))
    add("manifest a JSON list", _pack(None, good_plan, text=b"[1, 2]"))
    add("manifest NaN scale", _pack(None, good_plan, text=json.dumps(good).replace("0.02", "NaN").encode()))
    add("manifest Infinity scale", _pack(None, good_plan, text=json.dumps(good).replace("0.05", "Infinity").encode()))
    add("no input spec", _pack(_manifest(input=_DELETE), good_plan))
    add("input spec a list", _pack(_manifest(input=[1, 2]), good_plan))
    add("input shape differs", _pack(_manifest(**{"input/shape": [1, 4, 8, 4]}), good_plan))
    add("input dtype differs", _pack(_manifest(**{"input/dtype": "|u1"}), good_plan))
    add("input dtype unknown", _pack(_manifest(**{"input/dtype": "not-a-dtype"}), good_plan))
    add("input shape an int", _pack(_manifest(**{"input/shape": 7}), good_plan))
    add("input scale 0", _pack(_manifest(**{"input/quantization/scale": 0}), good_plan))
    add("input scale negative", _pack(_manifest(**{"input/quantization/scale": -1.0}), good_plan))
    add("input scale a string", _pack(_manifest(**{"input/quantization/scale": "x"}), good_plan))
    add("input zero point 128", _pack(_manifest(**{"input/quantization/zero_point": 128}), good_plan))
    add("input zero point -129", _pack(_manifest(**{"input/quantization/zero_point": -129}), good_plan))
    add("input zero point a float", _pack(_manifest(**{"input/quantization/zero_point": 1.0}), good_plan))
    add("input zero point a bool", _pack(_manifest(**{"input/quantization/zero_point": True}), good_plan))
    add("input without quantization", _pack(_manifest(**{"input/quantization": _DELETE}), good_plan))
    add("output quantization missing zero point",
        _pack(_manifest(**{"output/quantization/zero_point": _DELETE}), good_plan))
    # packed output views
    add("no packed outputs", _pack(_manifest(outputs=_DELETE), good_plan))
    add("outputs not a list", _pack(_manifest(outputs={"a": 1}), good_plan))
    add("outputs empty", _pack(_manifest(outputs=[]), good_plan))
    views33 = [{"name": f"v{i}", "shape": [1], "dtype": "|i1", "bytes": 1, "packed_offset": i} for i in range(33)]
    add("33 output views", _pack(_manifest(outputs=views33), good_plan))
    add("duplicate view name", _pack(_manifest(**{"outputs/1/name": "boxes"}), good_plan))
    add("view name not a string", _pack(_manifest(**{"outputs/0/name": 5}), good_plan))
    add("view rank 5", _pack(_manifest(**{"outputs/0/shape": [1, 1, 2, 2, 2]}), good_plan))
    add("view dimension 0", _pack(_manifest(**{"outputs/0/shape": [0, 8]}), good_plan))
    add("view dimension a float", _pack(_manifest(**{"outputs/0/shape": [2.0, 4]}), good_plan))
    add("view dtype float32", _pack(_manifest(**{"outputs/0/dtype": "<f4"}), good_plan))
    add("view bytes differ", _pack(_manifest(**{"outputs/0/bytes": 9}), good_plan))
    add("view offset wrong", _pack(_manifest(**{"outputs/1/packed_offset": 9}), good_plan))
    add("views do not cover the output", _pack(_manifest(**{"outputs/1/shape": [119], "outputs/1/bytes": 119}),
                                               good_plan))
    add("view dequantize without quantization",
        _pack(_manifest(**{"outputs/0/quantization": _DELETE}), good_plan))
    add("view dequantize with scale 0", _pack(_manifest(**{"outputs/0/quantization/scale": 0.0}), good_plan))
    add("view quantization zero point 255 on u1",
        _pack(_manifest(**{"outputs/1/quantization": {"scale": 1.0, "zero_point": 255}}), good_plan))
    add("view quantization zero point 256 on u1",
        _pack(_manifest(**{"outputs/1/quantization": {"scale": 1.0, "zero_point": 256}}), good_plan))
    add("view without name", _pack(_manifest(**{"outputs/0/name": _DELETE}), good_plan))
    add("view a list", _pack(_manifest(**{"outputs/0": [1, 2]}), good_plan))
    # plan header and tensor records
    for label, kw in [("plan magic", {"header_edits": {0: 0x55474E30}}), ("plan version 1", {"version": 1}),
                      ("plan version 3", {"version": 3}), ("plan version 4", {"version": 4}),
                      ("tensor count 0", {"header_edits": {2: 0}}), ("op count 0", {"header_edits": {3: 0}}),
                      ("arena 0", {"header_edits": {4: 0}}), ("arena over 16 MiB", {"header_edits": {4: 16 * 2 ** 20 + 1}}),
                      ("input index 3", {"header_edits": {5: 3}}), ("thread field 2", {"threads": 2}),
                      ("thread field 1", {"threads": 1}), ("plan with a trailing byte", {"trailing": 1}),
                      ("tensor type 5", {"tensor_edits": {(1, 2): 5}}), ("tensor rank 5", {"tensor_edits": {(0, 3): 5}}),
                      ("tensor dimension 0", {"tensor_edits": {(0, 5): 0}}),
                      ("tensor constant flag 2", {"tensor_edits": {(1, 8): 2}}),
                      ("tensor reserved word", {"tensor_edits": {(1, 10): 1}}),
                      ("tensor offset unaligned", {"tensor_edits": {(2, 0): 2433}}),
                      ("tensor offsets out of order", {"tensor_edits": {(2, 0): 128}}),
                      ("tensor past the arena", {"tensor_edits": {(2, 0): 2560}}),
                      ("tensor byte count", {"tensor_edits": {(0, 1): 127}}),
                      ("input tensor constant", {"input_const": 1}),
                      ("float32 output with packed views", {"out_type": 1})]:
        plan = _plan(**kw)
        add(label, _pack(good, plan))
    add("float32 output without packed views",
        _pack(_manifest(outputs=_DELETE, **{"output/dtype": "<f4", "output/quantization": _DELETE}), _plan(out_type=1)))
    return out


def sha(blob):
    return hashlib.sha256(blob).hexdigest()


def verdict(load, path, InvalidBundle):
    """'ok', 'InvalidBundle' or the name of any other exception type `load(path)` raised."""
    try:
        model = load(path)
    except InvalidBundle:
        return "InvalidBundle"
    except Exception as exc:  # noqa: BLE001 -- the class is the verdict
        return type(exc).__name__
    md = model.metadata
    return "ok:" + json.dumps({"in": list(md["input"]["shape"]), "out_bytes": md["output"]["bytes"],
                               "views": [v["name"] for v in md.get("outputs", [])],
                               "threads": md["dsp_threads"], "plan_bytes": md["plan_bytes"]}, sort_keys=True)

