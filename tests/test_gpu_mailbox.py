"""Session pipeline mode 1, the reference's "mailbox" (runtime/bridge.c:161-184): a resident
CUDA graph per session that copies a pinned input slot in, runs the network and copies the output
slot out. Results equal the blocking mode's and the reference's, across successive calls, with
profiling switched on and off, and after the input table changes."""
import ctypes as C

import numpy as np
import pytest

from conftest import model_path

pytestmark = pytest.mark.gpu


class Mailbox:
    def __init__(self, lib, plan, pipeline):
        self.lib, self.buf = lib, C.create_string_buffer(plan, len(plan))
        err = C.c_int()
        self.h = lib.ug_open_mode(self.buf, len(plan), pipeline, C.byref(err))
        assert self.h, (err.value, lib.ug_last_error())
        import struct
        inp, out = struct.unpack_from("<2I", plan, 20)
        self.ni = struct.unpack_from("<12I", plan, 32 + 48 * inp)[1]
        self.no = struct.unpack_from("<12I", plan, 32 + 48 * out)[1]

    def infer(self, x, ni=None):
        y = np.empty(self.no, dtype=np.int8)
        x = np.ascontiguousarray(x).reshape(-1)
        rc = self.lib.ug_infer(self.h, x.ctypes.data, ni or self.ni, y.ctypes.data, self.no)
        assert rc == 0, (rc, self.lib.ug_last_error())
        return y

    def close(self):
        self.lib.ug_close(self.h)


def seeded(shape, seed):
    return np.random.default_rng(seed).integers(-128, 128, size=shape, dtype=np.int64).astype(np.int8)


def test_mailbox_matches_blocking_and_reference(native, golden_models):
    from unoq_dsp import load
    plan = load(model_path("mobilenetv4-small")).plan
    xs = [seeded((1, 224, 224, 3), s) for s in (0, 1, 2, 3)]
    blocking = Mailbox(native, plan, 0)
    try:
        want = [blocking.infer(x) for x in xs]
    finally:
        blocking.close()
    m = Mailbox(native, plan, 1)
    try:
        for _ in range(2):  # successive calls reuse the resident graph and slots
            got = [m.infer(x) for x in xs]
            for g, w in zip(got, want):
                np.testing.assert_array_equal(g, w)
        np.testing.assert_array_equal(got[0], golden_models["mobilenetv4-small/y0"])
        np.testing.assert_array_equal(got[1], golden_models["mobilenetv4-small/y1"])
        out = np.empty(16, dtype=np.int8)
        assert native.ug_snapshot_tensor(m.h, 0, out.ctypes.data, 16) == 1003  # bridge.c:128
        counters = (C.c_uint64 * 130)()
        assert native.ug_profile_control(m.h, 1, counters, C.sizeof(counters)) == 0
        np.testing.assert_array_equal(m.infer(xs[2]), want[2])  # profiled: the ordinary path
        assert native.ug_profile_control(m.h, 2, counters, C.sizeof(counters)) == 0
        assert counters[0] == 1
        assert native.ug_profile_control(m.h, 0, counters, C.sizeof(counters)) == 0
        np.testing.assert_array_equal(m.infer(xs[3]), want[3])
        assert native.ug_last_infer_ms(m.h) > 0
        assert native.ug_infer(m.h, xs[0].ctypes.data, m.ni - 1, out.ctypes.data, m.no) == 1003
    finally:
        m.close()


def test_mailbox_with_an_input_table(native):
    """The byte table of the image APIs on the device: the mailbox graph is rebuilt when the table
    changes and lands uint8 pixels through it."""
    from unoq_dsp import load
    plan = load(model_path("mobilenetv4-small")).plan
    table = np.random.default_rng(4).integers(-128, 128, size=(256, 3), dtype=np.int64).astype(np.int8)
    pixels = np.random.default_rng(5).integers(0, 256, size=(224, 224, 3), dtype=np.int64).astype(np.uint8)
    mapped = table[pixels, np.arange(3)]
    outs = []
    for pipeline in (0, 1):
        s = Mailbox(native, plan, pipeline)
        try:
            plain = s.infer(mapped)
            assert native.ug_set_input_table(s.h, table.ctypes.data, 3) == 0
            via_table = s.infer(pixels)
            assert native.ug_set_input_table(s.h, None, 0) == 0
            np.testing.assert_array_equal(s.infer(mapped), plain)
        finally:
            s.close()
        np.testing.assert_array_equal(via_table, plain)
        outs.append(plain)
    np.testing.assert_array_equal(outs[0], outs[1])
