"""CPU: the .uqmodel loader (unoq_dsp.bundle) against the reference loader's verdicts on 73
seeded files (tests/golden/bundle_cases.py, verdicts in bundle.json from
make_bundle_golden.py): every file the reference accepts loads here with the same manifest
summary, every file it rejects raises InvalidBundle here."""
import json
import sys

import pytest

from conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
import bundle_cases  # noqa: E402

GOLD = json.loads((GOLDEN / "bundle.json").read_text())


def test_corpus_is_regenerated_identically():
    cases = bundle_cases.cases()
    assert [c[0] for c in cases] == [g["label"] for g in GOLD]
    for (label, blob), g in zip(cases, GOLD):
        assert bundle_cases.sha(blob) == g["sha256"], label


@pytest.mark.parametrize("index", range(len(GOLD)), ids=[g["label"] for g in GOLD])
def test_loader_matches_reference_verdict(index, tmp_path):
    from unoq_dsp.bundle import load
    from unoq_dsp.errors import InvalidBundle
    label, blob = bundle_cases.cases()[index]
    path = tmp_path / "case.uqmodel"
    path.write_bytes(blob)
    assert bundle_cases.verdict(load, path, InvalidBundle) == GOLD[index]["verdict"], label


def test_save_round_trip(tmp_path):
    from unoq_dsp.bundle import CompiledModel, load
    from unoq_dsp.errors import InvalidBundle
    label, blob = bundle_cases.cases()[0]
    src = tmp_path / "a.uqmodel"
    src.write_bytes(blob)
    model = load(src)
    dst = tmp_path / "b.uqmodel"
    model.save(dst)
    again = load(dst)
    assert again.plan == model.plan and again.metadata["outputs"][1]["name"] == "scores"
    bad = CompiledModel(model.plan, dict(model.metadata, input=dict(model.metadata["input"], shape=(1, 2))))
    with pytest.raises(InvalidBundle):
        bad.save(tmp_path / "c.uqmodel")
