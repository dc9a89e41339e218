"""The product's requantisation constants (csrc/requant.cuh, used by every conv and depthwise
epilogue) against the oracle's `scale` (runtime/qnn.c:61-83): 2.56 M edge-dense cases, including
accumulators next to the tie cut, every shift in [-31, 15] and the kRelu short form."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="nvcc not on PATH")
def test_requant_form_matches_reference_scale(tmp_path):
    lib = ROOT / "oracle" / "liboracle.so"
    if not lib.is_file():
        subprocess.run(["make", "-C", str(ROOT / "oracle")], check=True, stdout=subprocess.DEVNULL)
    exe = tmp_path / "requant_form"
    subprocess.run(["nvcc", "-std=c++17", "-O2", "-I", str(ROOT / "unoq-dsp_b200" / "csrc"),
                    str(ROOT / "tests" / "native" / "requant_form.cu"), "-L", str(lib.parent), "-loracle",
                    f"-Xlinker=-rpath,{lib.parent}", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout + out.stderr
    assert " mismatches 0 fast_mismatches 0" in out.stdout
