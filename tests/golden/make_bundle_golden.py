"""Record the REFERENCE package's verdict on every seeded .uqmodel of bundle_cases.py.

Run where the reference checkout is mounted (UNOQ_REFERENCE_DIR, default: a `reference`
directory beside this repository):

    python tests/golden/make_bundle_golden.py

The reference's src/unoq_dsp/bundle.py is imported in a separate interpreter (so its package does
not clash with this repository's). Writes bundle.json: per case its label, the SHA-256 of the file
bytes and the verdict -- "ok:<summary of the loaded manifest>", "InvalidBundle" or another
exception class name. tests/test_bundle.py regenerates the files and requires the same verdicts
from unoq_dsp.bundle.load.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_SRC = Path(os.environ.get("UNOQ_REFERENCE_DIR", HERE.parents[2] / "reference")) / "src"

WORKER = r'''
import json, sys, tempfile, os
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[2])
from unoq_dsp.bundle import load
from unoq_dsp.errors import InvalidBundle
import bundle_cases as bc
out = []
with tempfile.TemporaryDirectory() as d:
    for label, blob in bc.cases():
        path = os.path.join(d, "case.uqmodel")
        with open(path, "wb") as f:
            f.write(blob)
        out.append({"label": label, "sha256": bc.sha(blob), "verdict": bc.verdict(load, path, InvalidBundle)})
print(json.dumps(out))
'''


def main():
    res = subprocess.run([sys.executable, "-c", WORKER, str(REF_SRC), str(HERE)], capture_output=True, text=True,
                         check=True)
    cases = json.loads(res.stdout)
    (HERE / "bundle.json").write_text(json.dumps(cases, indent=1) + "\n")
    print(f"wrote {len(cases)} verdicts:", sum(c["verdict"].startswith("ok") for c in cases), "accepted")


if __name__ == "__main__":
    main()
