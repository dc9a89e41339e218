"""TEST INFRASTRUCTURE ONLY: ctypes front ends for the two CPU parity checkers.

* ``Oracle``    -- liboracle.so, the scalar C restatement in uq_oracle.c.
* ``Reference`` -- oracle/_ref/libug_ref.so, the reference runtime's own graph.c/qnn.c/gemm.c
  compiled for the host from its sources (see oracle/Makefile). It exports the reference's
  process-global ``ug_load``/``ug_run`` ABI (runtime/graph.h:39-45).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline / reference legs use these,
and only as checkers or as the timed CPU baseline. The product never imports this module.
"""
import ctypes as C
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libug_ref.so"
REF_PLAIN_LIB = HERE / "_ref" / "libug_ref_plain.so"


def _bytes(plan):
    plan = bytes(plan)
    return plan, C.create_string_buffer(plan, len(plan))


class Oracle:
    """The C restatement: stateless, runs any number of images per call."""

    def __init__(self, path=ORACLE_LIB):
        self.lib = C.CDLL(str(path))
        self.lib.uqo_run.argtypes = [C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p, C.c_uint32]
        self.lib.uqo_run.restype = C.c_int
        for name in ("uqo_input_bytes", "uqo_output_bytes"):
            getattr(self.lib, name).argtypes = [C.c_void_p, C.c_uint32]
            getattr(self.lib, name).restype = C.c_uint32
        self.lib.uqo_scale.argtypes = [C.c_int32, C.c_int32, C.c_int]
        self.lib.uqo_scale.restype = C.c_int32

    def run(self, plan, x, images=1):
        plan, buf = _bytes(plan)
        ni = self.lib.uqo_input_bytes(buf, len(plan))
        no = self.lib.uqo_output_bytes(buf, len(plan))
        x = np.ascontiguousarray(x)
        if x.nbytes != ni * images:
            raise ValueError(f"expected {ni * images} input bytes, got {x.nbytes}")
        y = np.empty(no * images, dtype=np.int8)
        rc = self.lib.uqo_run(buf, len(plan), x.ctypes.data, y.ctypes.data, images)
        if rc:
            raise RuntimeError(f"oracle rc={rc}")
        return y

    def scale(self, v, m, shift):
        return self.lib.uqo_scale(int(v), int(m), int(shift))


class Reference:
    """The reference runtime built from its own C sources (one global graph per process)."""

    def __init__(self, path=REF_LIB):
        if not Path(path).is_file():
            raise FileNotFoundError(f"{path} missing: run `make -C oracle ref` where the reference is mounted")
        # RTLD_LOCAL with a private handle: the flag and plain builds keep separate globals.
        self.lib = C.CDLL(str(path), mode=C.RTLD_LOCAL)
        self.lib.ug_load.argtypes = [C.c_void_p, C.c_uint32]
        self.lib.ug_run.argtypes = [C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32]
        self.lib.ug_input_bytes.restype = C.c_uint32
        self.lib.ug_output_bytes.restype = C.c_uint32
        self._plan = None

    def load(self, plan):
        plan, buf = _bytes(plan)
        self._buf = buf
        rc = self.lib.ug_load(buf, len(plan))
        self._plan = plan if rc == 0 else None
        return rc

    def run(self, plan, x, images=1):
        if self._plan != bytes(plan):
            rc = self.load(plan)
            if rc:
                raise RuntimeError(f"reference ug_load rc={rc}")
        ni, no = self.lib.ug_input_bytes(), self.lib.ug_output_bytes()
        x = np.ascontiguousarray(x).reshape(-1).view(np.uint8)
        if x.nbytes != ni * images:
            raise ValueError(f"expected {ni * images} input bytes, got {x.nbytes}")
        y = np.empty(no * images, dtype=np.int8)
        for i in range(images):
            xi = np.ascontiguousarray(x[i * ni:(i + 1) * ni])
            yi = y[i * no:(i + 1) * no]
            rc = self.lib.ug_run(xi.ctypes.data, ni, yi.ctypes.data, no)
            if rc:
                raise RuntimeError(f"reference ug_run rc={rc}")
        return y


def available():
    return {"oracle": ORACLE_LIB.is_file(), "reference": REF_LIB.is_file()}
