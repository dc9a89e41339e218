"""Failure detection on the GPU without a fault: a device-side wait that runs out.

Every wait of the tensor-core conv kernels is bounded (about 2 s of SM cycles); on expiry the
kernel records a site code, drains its MMAs and copies, frees TMEM and exits, and the host
reports 2003. The test-only switch UNOQ_FAULT_WITHHOLD_COMMIT=1, read when a plan is loaded, makes
the MMA thread of one CTA never signal its first accumulator, so that CTA's epilogue wait runs
out (a flag that nothing sets). The run must return 2003, unload the graph as any failed run does
(the reference's ready = 0, runtime/graph.c:298-305), and a reload without the switch must run
clean on the same device and context."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _load(native, plan):
    buf = C.create_string_buffer(plan, len(plan))
    assert native.ug_load(buf, len(plan)) == 0, native.ug_last_error()
    return buf


def _run(native, x):
    y = np.empty(native.ug_output_bytes(), dtype=np.int8)
    rc = native.ug_run(x.ctypes.data, x.nbytes, y.ctypes.data, y.nbytes)
    return rc, y


def test_device_wait_timeout_reports_2003_then_reload_runs_clean(native, golden_ops, monkeypatch):
    plan, x = golden_ops["conv_pw_c0/plan"].tobytes(), golden_ops["conv_pw_c0/x"]
    monkeypatch.setenv("UNOQ_FAULT_WITHHOLD_COMMIT", "1")
    keep = _load(native, plan)  # noqa: F841
    rc, _ = _run(native, x)
    assert rc == 2003, (rc, native.ug_last_error())
    assert b"timed out" in native.ug_last_error()
    assert native.ug_input_bytes() == 0  # the failed run unloaded the graph
    monkeypatch.delenv("UNOQ_FAULT_WITHHOLD_COMMIT")
    keep = _load(native, plan)  # noqa: F841
    rc, y = _run(native, x)
    assert rc == 0, native.ug_last_error()
    np.testing.assert_array_equal(y, golden_ops["conv_pw_c0/y"])


def test_session_survives_a_timed_out_call(native, golden_ops, monkeypatch):
    """Sessions keep their plan after a failed call (bridge.c passes the code through): the next
    call on a session loaded without the switch is exact."""
    from gpuhelp import NativeSession
    plan, x = golden_ops["conv_pw_c0/plan"].tobytes(), golden_ops["conv_pw_c0/x"]
    monkeypatch.setenv("UNOQ_FAULT_WITHHOLD_COMMIT", "1")
    with NativeSession(native, plan) as s:
        y = np.empty(s.no, dtype=np.int8)
        assert native.ug_infer(s.handle, x.ctypes.data, s.ni, y.ctypes.data, s.no) == 2003
    monkeypatch.delenv("UNOQ_FAULT_WITHHOLD_COMMIT")
    with NativeSession(native, plan) as s:
        np.testing.assert_array_equal(s.run(x), golden_ops["conv_pw_c0/y"])
