"""CPU: the GPU decoder's inputs and host finish. YOLODecoder.device_config's tables must give the
host decoder's own float32 scores and distances for every int8 code, and the decoder contract
(tests/decode_emulation.py) followed by YOLODecoder.finish must reproduce YOLODecoder.decode
exactly, ties included. The kernel itself is checked against the same contract on the GPU."""
import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import decode_cases as dc  # noqa: E402
from decode_emulation import emulate, pack, packed_specs  # noqa: E402
from unoq_dsp.modern import YOLODecoder  # noqa: E402


def contract():
    task, outputs, shape = dc.yolo_contract()
    specs, total = packed_specs(outputs)
    return YOLODecoder(task, specs, shape), specs, total


def skewed_raw(specs, rng, hot=0.004, lo=-128, hi=-60):
    raw = {}
    for spec in specs:
        if spec["shape"][-1] == 4:
            raw[spec["name"]] = rng.integers(-128, 128, size=spec["shape"]).astype(np.int8)
        else:
            v = rng.integers(lo, hi, size=spec["shape"])
            mask = rng.random(spec["shape"]) < hot
            v[mask] = rng.integers(100, 128, size=int(mask.sum()))
            raw[spec["name"]] = v.astype(np.int8)
    return raw


def test_tables_reproduce_the_host_decoder_values():
    decoder, specs, _ = contract()
    config = decoder.device_config()
    rng = np.random.default_rng(5)
    for level in range(3):
        lv = config.level[level]
        box, score = decoder.names[2 * level], decoder.names[2 * level + 1]
        raw = {box: rng.integers(-128, 128, size=decoder.specs[box]["shape"]).astype(np.int8),
               score: rng.integers(-128, 128, size=decoder.specs[score]["shape"]).astype(np.int8)}
        logits = decoder._dequantised(raw, score)
        host = 1 / (1 + np.exp(-np.clip(logits.reshape(-1, decoder.classes), -80, 80)))
        table = np.array(lv.score[:], dtype="f4")[raw[score][0].reshape(-1, decoder.classes).astype(np.int64) + 128]
        np.testing.assert_array_equal(table.view(np.uint32), host.view(np.uint32))
        dist = np.array(lv.distance[:], dtype="f4")[raw[box][0].astype(np.int64) + 128]
        np.testing.assert_array_equal(dist.view(np.uint32), decoder._dequantised(raw, box).view(np.uint32))
    # order codes: same order as the scores, equal scores share a code
    s = np.concatenate([np.array(config.level[l].score[:], dtype="f4") for l in range(3)])
    r = np.concatenate([np.array(config.level[l].rank[:]) for l in range(3)])
    i, j = np.triu_indices(len(s), 1)
    assert np.array_equal(np.sign(s[i] - s[j]), np.sign(r[i].astype(int) - r[j].astype(int)))
    assert r.max() < 1024 and (lv.box_offset, lv.score_offset) == (decoder.specs[decoder.names[4]]["packed_offset"],
                                                                    decoder.specs[decoder.names[5]]["packed_offset"])


@pytest.mark.parametrize("seed", range(6))
def test_contract_then_finish_equals_host_decode(seed):
    decoder, specs, total = contract()
    config = decoder.device_config()
    rng = np.random.default_rng(seed)
    # dense ties: few distinct logits (seed 0/1), the golden cases' mix, a flat head (seed 5)
    raw = [skewed_raw(specs, rng, hot=0.0, lo=-100, hi=-97), skewed_raw(specs, rng, hot=0.5, lo=-128, hi=-127),
           skewed_raw(specs, rng), skewed_raw(specs, rng, hot=0.02, lo=-128, hi=127),
           skewed_raw(specs, rng, hot=0.3), skewed_raw(specs, rng, hot=0.0, lo=-90, hi=-89)][seed]
    geometry = {"ratio": .5, "left": 3, "top": 40, "width": 640, "height": 480}
    for options in ({}, {"score_threshold": 0.0, "max_results": 300}, {"max_results": 1}, {"score_threshold": .3}):
        k = decoder.check_options(**options)
        records = emulate(config, pack(raw, specs, total)[None], k)[0]
        got = decoder.finish(records, geometry=geometry, **options)
        assert got == decoder.decode(raw, geometry=geometry, **options)


def test_golden_cases_through_the_contract():
    decoder, specs, total = contract()
    config = decoder.device_config()
    for raw, geometry, options in dc.yolo_cases(specs):
        records = emulate(config, pack(raw, specs, total)[None], decoder.check_options(**options))[0]
        assert decoder.finish(records, geometry=geometry, **options) == decoder.decode(raw, geometry=geometry, **options)


def test_finish_checks_options_like_decode():
    decoder, _, _ = contract()
    with pytest.raises(ValueError):
        decoder.finish([], geometry={}, iou_threshold=.5)
    with pytest.raises(ValueError):
        decoder.finish([], geometry={}, max_results=301)
