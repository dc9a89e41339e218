"""CPU: the operator ABI's host-only entry point uq_validate (include/unoq_ops.h) against the
reference's own uq_validate (runtime/qnn.c:209-252, in oracle/_ref/libug_ref.so): identical codes
and work on every one-op conv / depthwise / pool / softmax-table case and on corrupted parameter
blocks; and the header-level ug_dot_u8i8 contract (runtime/kernels.h:7)."""
import ctypes as C

import numpy as np
import pytest

from conftest import GOLDEN
from opabi import Plan, bind, reference_lib

GOLD = np.load(GOLDEN / "ops.npz")


def _cases():
    out = []
    for n in sorted({k.split("/")[0] for k in GOLD.files}):
        p = Plan(GOLD[f"{n}/plan"].tobytes())
        if p.no == 1 and 14 <= p.ops[0].code <= 17:
            out.append(n)
    return out


def _corruptions(q, code):
    """(label, q') variants that the loader rejects or accepts at its edges."""
    yield "as is", q
    for idx, val, label in [(12, 128, "input zero point above 127"), (14, 10, "min above max"), (19, 2, "flags"),
                            (0, 0, "kernel height 0"), (10, 999, "output height")]:
        v = q.copy()
        if label == "min above max":
            v[14], v[15] = 10, 5
        else:
            v[idx] = val
        yield label, v
    if code in (14, 15):
        oc = int(q[17])
        v = q.copy()
        v[20 + oc] = -1
        yield "negative multiplier", v
        v = q.copy()
        v[20 + 2 * oc] = 16
        yield "shift above 15", v
        v = q.copy()
        v[20] = 2 ** 31 - 1
        yield "bias that overflows the accumulator bound", v


@pytest.mark.parametrize("name", _cases())
def test_uq_validate_matches_reference(name, native):
    ref = reference_lib()
    if ref is None:
        pytest.skip("oracle/_ref/libug_ref.so not built")
    ours = bind(native)
    plan = Plan(GOLD[f"{name}/plan"].tobytes())
    o = plan.ops[0]
    a, b, z, t = (plan.tensors[i] for i in (o.a, o.b, o.out, o.p[0]))
    q0 = plan.data(o.p[0]).view(np.int32).copy()
    w = plan.data(o.b).view(np.int8).copy()
    for label, q in _corruptions(q0, o.code):
        got = []
        for lib in (ref, ours):
            work = C.c_uint64(7)
            rc = lib.uq_validate(C.byref(o), C.byref(a), C.byref(b), C.byref(z), C.byref(t), q.ctypes.data,
                                 w.ctypes.data, C.byref(work))
            got.append((rc, work.value))
        assert got[0] == got[1], (label, got)


def test_uq_validate_refuses_null(native):
    ours = bind(native)
    plan = Plan(GOLD["conv_pw_c0/plan"].tobytes())
    o = plan.ops[0]
    a, b, z, t = (plan.tensors[i] for i in (o.a, o.b, o.out, o.p[0]))
    q = plan.data(o.p[0]).view(np.int32).copy()
    work = C.c_uint64(0)
    assert ours.uq_validate(C.byref(o), C.byref(a), C.byref(b), C.byref(z), C.byref(t), q.ctypes.data, None,
                            C.byref(work)) == 22


def test_ug_dot_u8i8_header_contract(tmp_path):
    """The static inline ug_dot_u8i8 of include/unoq_ops.h compiles as C and equals the scalar sum."""
    import shutil
    import subprocess
    from conftest import ROOT
    cc = shutil.which("gcc")
    if cc is None:
        pytest.skip("gcc not on PATH")
    src = tmp_path / "dot.c"
    src.write_text('#include "unoq_ops.h"\n#include <stdio.h>\nint main(void){uint8_t x[37];int8_t w[37];'
                   'for(int i=0;i<37;i++){x[i]=(uint8_t)(i*53+200);w[i]=(int8_t)(i*31-90);}'
                   'printf("%d\\n",ug_dot_u8i8(x,w,37));return 0;}\n')
    exe = tmp_path / "dot"
    subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-I", str(ROOT / "include"), str(src), "-o", str(exe)],
                   check=True)
    out = int(subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout)
    x = np.array([(i * 53 + 200) % 256 for i in range(37)], dtype=np.int64)
    w = np.array([((i * 31 - 90 + 128) % 256) - 128 for i in range(37)], dtype=np.int64)
    assert out == int((x * w).sum())
