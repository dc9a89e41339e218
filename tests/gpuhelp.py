"""Helpers for GPU parity tests: drive libunoq_cuda.so through its C ABI with ctypes."""
import ctypes as C

import numpy as np


class NativeSession:
    """ug_open_mode / ug_infer / ug_infer_batch / ug_close on one plan."""

    def __init__(self, lib, plan):
        self.lib = lib
        self.plan = C.create_string_buffer(bytes(plan), len(plan))
        err = C.c_int()
        self.handle = lib.ug_open_mode(self.plan, len(plan), 0, C.byref(err))
        if not self.handle:
            raise RuntimeError(f"ug_open_mode failed: {err.value} {lib.ug_last_error()}")
        import struct
        magic, version, nt, no, arena, inp, out, flags = struct.unpack_from("<8I", plan)
        self.ni = struct.unpack_from("<12I", plan, 32 + 48 * inp)[1]
        self.no = struct.unpack_from("<12I", plan, 32 + 48 * out)[1]

    def run(self, x, images=1):
        x = np.ascontiguousarray(x).reshape(-1).view(np.int8)
        assert x.nbytes == self.ni * images
        y = np.empty(self.no * images, dtype=np.int8)
        if images == 1:
            rc = self.lib.ug_infer(self.handle, x.ctypes.data, self.ni, y.ctypes.data, self.no)
        else:
            rc = self.lib.ug_infer_batch(self.handle, x.ctypes.data, images, y.ctypes.data)
        if rc:
            raise RuntimeError(f"inference rc={rc} {self.lib.ug_last_error()}")
        return y

    def close(self):
        if self.handle:
            self.lib.ug_close(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()
