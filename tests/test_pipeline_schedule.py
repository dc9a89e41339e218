"""The pipelined batch's piece schedule (csrc/engine.hpp): pieces cover the batch, and every rank
of a gathered run cuts the same pieces whatever growth each process learned on its own (a
divergent schedule makes the per-piece gather wait for a step its peer never enqueues)."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="nvcc not on PATH")
def test_joined_ranks_cut_identical_pieces(tmp_path):
    exe = tmp_path / "pipeline_pieces"
    csrc = ROOT / "unoq-dsp_b200" / "csrc"
    subprocess.run(["nvcc", "-std=c++17", "-O1", "-I", str(csrc), "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "native" / "pipeline_pieces.cu"), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout + out.stderr
    assert out.stdout.strip().endswith("ok")
