"""CPU: the C ABI library loads and exports its header; host-side logic without a GPU."""
import ctypes as C
import hashlib
import re
from pathlib import Path

import numpy as np
import pytest

import opcases
import plancorrupt
from conftest import ROOT, model_path


def declared_symbols():
    names = []
    for header in (ROOT / "include").glob("*.h"):
        names += re.findall(r"^UG_API\s+[\w\s\*]*?\b(\w+)\s*\(", header.read_text(), flags=re.M)
    return names


def test_library_exports_every_declared_symbol(native):
    names = declared_symbols()
    assert len(names) >= 24
    missing = [n for n in names if not hasattr(native, n)]
    assert not missing, missing


def test_reference_abi_names_present(native):
    # runtime/graph.h:39-45 and the bridge exports the reference's Python transport binds.
    for name in ("ug_load", "ug_run", "ug_input_bytes", "ug_output_bytes", "ug_snapshot", "ug_profile",
                 "ug_open_mode", "ug_open", "ug_infer", "ug_close", "ug_snapshot_tensor", "ug_profile_control"):
        assert hasattr(native, name), name


def test_loader_codes_match_reference(native):
    golden = np.load(ROOT / "tests" / "golden" / "codes.npz")
    for i, (label, plan) in enumerate(plancorrupt.variants()):
        assert hashlib.sha256(plan).digest() == golden[f"{i}/sha256"].tobytes(), label
        buf = C.create_string_buffer(plan, len(plan))
        assert native.ug_validate_plan(buf, len(plan)) == int(golden[f"{i}/code"][0]), label


def test_loader_accepts_every_op_case(native, golden_ops):
    for name, _ in opcases.all_cases(1):
        plan = golden_ops[f"{name}/plan"].tobytes()
        assert native.ug_validate_plan(C.create_string_buffer(plan, len(plan)), len(plan)) == 0, name


@pytest.mark.parametrize("name", ["mobilenetv4-small", "yolo26n-320"])
def test_bundled_models_load_and_validate(name, native):
    from unoq_dsp import load
    model = load(model_path(name))
    assert native.ug_validate_plan(C.create_string_buffer(model.plan, len(model.plan)), len(model.plan)) == 0
    kind = {"mobilenetv4-small": "image_classification", "yolo26n-320": "yolo_one_to_one"}[name]
    assert model.metadata["task"]["kind"] == kind
    assert len(model.plan) > 1_000_000


def test_bundle_checksum_and_roundtrip(tmp_path):
    from unoq_dsp import CompiledModel, InvalidBundle, load
    plan, _ = opcases.block_case(np.random.default_rng(0), hw=4)
    spec = {"shape": [1, 4, 4, 32], "dtype": "int8", "quantization": {"scale": 0.05, "zero_point": -3}}
    out = {"shape": [1, 4, 4, 32], "dtype": "int8"}
    path = tmp_path / "m.uqmodel"
    CompiledModel(plan, {"input": spec, "output": out, "macs": 1}).save(path)
    model = load(path)
    assert model.plan == plan and model.metadata["input"]["shape"] == (1, 4, 4, 32)
    raw = bytearray(path.read_bytes())
    raw[-1] ^= 1
    path.write_bytes(bytes(raw))
    with pytest.raises(InvalidBundle):
        load(path)


def test_session_requires_a_library(tmp_path):
    from unoq_dsp import DSPError, Session
    plan, _ = opcases.block_case(np.random.default_rng(0), hw=4)
    from unoq_dsp import CompiledModel
    model = CompiledModel(plan, {"input": {"shape": (1, 4, 4, 32), "dtype": "int8"},
                                 "output": {"shape": (1, 4, 4, 32), "dtype": "int8"}})
    with pytest.raises(DSPError):
        Session(model, library=tmp_path / "missing.so")


def test_pipeline_argument_is_checked():
    from unoq_dsp import CompiledModel, Session
    plan, _ = opcases.block_case(np.random.default_rng(0), hw=4)
    model = CompiledModel(plan, {"input": {"shape": (1, 4, 4, 32), "dtype": "int8"},
                                 "output": {"shape": (1, 4, 4, 32), "dtype": "int8"}})
    with pytest.raises(ValueError):
        Session(model, pipeline="fast")
