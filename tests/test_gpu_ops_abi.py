"""The operator-level ABI (include/unoq_ops.h) on the GPU against the same symbols of the reference
runtime built for the host (oracle/_ref/libug_ref.so: runtime/qnn.c uq_run / uq_add / uq_mean /
uq_mul / uq_bmm / uq_softmax_exact / uq_post_register, runtime/gemm.c ug_matmul_u8i8*), byte for
byte: ours on device buffers, the reference on host buffers, identical inputs. Includes the
config-1 depthwise sweep and the config-0 pointwise conv at batch 256 through uq_run, past the
reference graph's 16 MiB arena (runtime/graph.h:7)."""
import ctypes as C

import numpy as np
import pytest

import configcases
from conftest import GOLDEN
from opabi import Device, Plan, UGTensor, batched, bind, reference_lib

pytestmark = pytest.mark.gpu
GOLD = np.load(GOLDEN / "ops.npz")


def _vision_cases():
    names = sorted({k.split("/")[0] for k in GOLD.files})
    out = []
    for n in names:
        p = Plan(GOLD[f"{n}/plan"].tobytes())
        if p.no == 1 and 14 <= p.ops[0].code <= 17:
            out.append(n)
    return out


VISION = _vision_cases()


@pytest.fixture(scope="module")
def ref():
    lib = reference_lib()
    if lib is None:
        pytest.skip("oracle/_ref/libug_ref.so not built")
    return lib


@pytest.fixture(scope="module")
def ops(native):
    assert native.ug_set_device(0) == 0
    return bind(native)


@pytest.fixture
def dev():
    return Device()


def seeded(shape, seed, lo=-128, hi=128, dtype=np.int8):
    return np.random.default_rng(seed).integers(lo, hi, size=shape, dtype=np.int64).astype(dtype)


def op_parts(plan):
    """(code, a, z, w bytes or None, q int32, post table or None) of a one-op vision plan."""
    o = plan.ops[0]
    a, z = plan.tensors[o.a], plan.tensors[o.out]
    q = plan.data(o.p[0]).view(np.int32).copy()
    w = plan.data(o.b).view(np.int8).copy() if o.code in (14, 15) else None
    post = plan.data(o.p[1] - 1).copy() if o.p[1] else None
    return o.code, a, z, w, q, post


def ref_uq_run(ref, code, a, z, x, w, q, post):
    ref.uq_prepare_reset()
    ref.uq_post_reset()
    if post is not None:
        ref.uq_post_register(q.ctypes.data, post.ctypes.data)
    y = np.empty(z.bytes, dtype=np.int8)
    wp = w.ctypes.data if w is not None else x.ctypes.data
    rc = ref.uq_run(code, C.byref(a), C.byref(z), x.ctypes.data, wp, y.ctypes.data, q.ctypes.data, 1)
    ref.uq_post_reset()
    return rc, y


def our_uq_run(ops, dev, code, a, z, x, w, q, post, pad=0):
    ops.uq_post_reset()
    dq = dev.put(q)
    dw = dev.put(w) if w is not None else None
    dx = dev.put(x, pad)
    dy = dev.empty(z.bytes, pad)
    if post is not None:
        ops.uq_post_register(dq, dev.put(post))
    rc = ops.uq_run(code, C.byref(a), C.byref(z), dx, dw, dy, dq, 1)
    ops.uq_post_reset()
    return rc, dev.get(dy, z.bytes)


@pytest.mark.parametrize("name", VISION)
def test_uq_run_matches_reference(name, ops, ref, dev):
    """Every one-op conv / depthwise / pool / softmax-table case at batch 3 (the golden image and two
    more): same bytes as the reference's uq_run, and the first image equals the golden output."""
    code, a, z, w, q, post = op_parts(Plan(GOLD[f"{name}/plan"].tobytes()))
    images = 3
    x = np.concatenate([GOLD[f"{name}/x"], seeded(2 * a.bytes, 99)])
    a3, z3 = batched(a, images), batched(z, images)
    rc_ref, y_ref = ref_uq_run(ref, code, a3, z3, x, w, q, post)
    rc, y = our_uq_run(ops, dev, code, a3, z3, x, w, q, post)
    assert rc_ref == 0 and rc == 0, (rc_ref, rc, ops.ug_last_error())
    np.testing.assert_array_equal(y, y_ref)
    np.testing.assert_array_equal(y[:z.bytes], GOLD[f"{name}/y"])


@pytest.mark.parametrize("name", ["conv_pw_c0", "conv_3x3_s2", "dw3_s2_wide", "dw5_s1_post"])
@pytest.mark.parametrize("pad", [1, 16])
def test_uq_run_unaligned_buffers(name, pad, ops, ref, dev):
    """Operands that start 1 or 16 bytes into an allocation (staged through aligned buffers)."""
    code, a, z, w, q, post = op_parts(Plan(GOLD[f"{name}/plan"].tobytes()))
    x = GOLD[f"{name}/x"]
    rc, y = our_uq_run(ops, dev, code, a, z, x, w, q, post, pad=pad)
    assert rc == 0, ops.ug_last_error()
    np.testing.assert_array_equal(y, GOLD[f"{name}/y"])


CONFIG_BATCH = [("config0_pw", 64)] + [(n, 256) for n, _ in configcases.config_cases()
                                       if n.startswith("config1") and ("dw3_s1" in n or "dw5_s2" in n)] + \
               [(n, 8) for n, _ in configcases.config_cases() if n.startswith("config1") and
                ("dw3_s2" in n or "dw5_s1" in n)]


@pytest.mark.parametrize("name,images", CONFIG_BATCH)
def test_config_layers_past_the_arena(name, images, ops, ref, dev):
    """BASELINE configs 0 and 1 as single ops at large batch through uq_run (batch 256 of a
    112x112x32 layer is 102 MB of input, beyond any reference plan)."""
    plan, xs, _ = configcases.build(name)
    code, a, z, w, q, post = op_parts(Plan(plan))
    an, zn = batched(a, images), batched(z, images)
    x = seeded(an.bytes, 7)
    rc_ref, y_ref = ref_uq_run(ref, code, an, zn, x, w, q, post)
    rc, y = our_uq_run(ops, dev, code, an, zn, x, w, q, post)
    assert rc_ref == 0 and rc == 0, (rc_ref, rc, ops.ug_last_error())
    bad = np.flatnonzero((y != y_ref).reshape(images, -1).any(axis=1))
    assert bad.size == 0, f"{bad.size} of {images} images differ, first {bad[:8].tolist()}"


def test_uq_run_refuses_bad_calls(ops, dev):
    code, a, z, w, q, post = op_parts(Plan(GOLD["conv_pw_c0/plan"].tobytes()))
    x = GOLD["conv_pw_c0/x"]
    dq, dw, dx, dy = dev.put(q), dev.put(w), dev.put(x), dev.empty(z.bytes)
    # host pointers where device memory is required
    assert ops.uq_run(code, C.byref(a), C.byref(z), x.ctypes.data, dw, dy, dq, 1) == 22
    assert ops.uq_run(5, C.byref(a), C.byref(z), dx, dw, dy, dq, 1) == 19
    bad = q.copy()
    bad[20 + 2 * bad[17]] = 40  # a shift above 15 (qnn.c:240)
    assert ops.uq_run(code, C.byref(a), C.byref(z), dx, dw, dy, dev.put(bad), 1) == 18
    zb = UGTensor.from_buffer_copy(bytes(z))
    zb.d[0] = 2  # batch axes disagree
    assert ops.uq_run(code, C.byref(a), C.byref(zb), dx, dw, dy, dq, 1) == 18
    assert ops.uq_run(code, C.byref(a), C.byref(z), dx, dw, dy, dq, 1) == 0  # still usable


def _op_case(name):
    plan = Plan(GOLD[f"{name}/plan"].tobytes())
    o = [op for op in plan.ops if op.code in (18, 24, 25, 27, 28)][-1]
    return plan, o


@pytest.mark.parametrize("name", ["add", "mul"])
def test_elementwise_binary(name, ops, ref, dev):
    plan, o = _op_case(name)
    q = plan.data(o.p[0]).view(np.int32).copy()
    count = plan.tensors[o.out].bytes * 5
    x, b = seeded(count, 1), seeded(count, 2)
    fn = "uq_add" if o.code == 18 else "uq_mul"
    y_ref = np.empty(count, dtype=np.int8)
    getattr(ref, fn)(x.ctypes.data, b.ctypes.data, y_ref.ctypes.data, count, q.ctypes.data)
    dy = dev.empty(count)
    getattr(ops, fn)(dev.put(x), dev.put(b), dy, count, dev.put(q))
    assert ops.uq_status() == 0, ops.ug_last_error()
    np.testing.assert_array_equal(dev.get(dy, count), y_ref)


def test_mean(ops, ref, dev):
    plan, o = _op_case("mean")
    q = plan.data(o.b).view(np.int32).copy()
    a = plan.tensors[o.a]
    batches, channels = 6, a.d[3]
    x = seeded(batches * a.d[1] * a.d[2] * channels, 3)
    y_ref = np.empty(batches * channels, dtype=np.int8)
    ref.uq_mean(x.ctypes.data, y_ref.ctypes.data, batches, channels, q.ctypes.data)
    dy = dev.empty(batches * channels)
    ops.uq_mean(dev.put(x), dy, batches, channels, dev.put(q))
    assert ops.uq_status() == 0, ops.ug_last_error()
    np.testing.assert_array_equal(dev.get(dy, batches * channels), y_ref)


def test_softmax_exact(ops, ref, dev, native):
    plan, o = _op_case("softmax_exact")
    q = plan.data(o.b).view(np.int32).copy()
    width = int(q[0])
    nbytes = plan.tensors[o.a].bytes * 4
    x = seeded(nbytes, 4)
    y_ref = np.empty(nbytes, dtype=np.int8)
    ref.uq_softmax_exact(x.ctypes.data, y_ref.ctypes.data, nbytes, q.ctypes.data)
    dy, dx, dq = dev.empty(nbytes), dev.put(x), dev.put(q)
    np.testing.assert_array_equal(dev.get(dx, nbytes), x)  # the device copies hold what was put
    np.testing.assert_array_equal(dev.get(dq, q.nbytes, np.int32), q)
    ops.uq_softmax_exact(dx, dy, nbytes, dq)
    assert ops.uq_status() == 0, ops.ug_last_error()
    got = dev.get(dy, nbytes)
    dy2 = dev.empty(nbytes)
    ops.uq_softmax_exact(dx, dy2, nbytes, dq)
    again = dev.get(dy2, nbytes)
    assert np.array_equal(got, again), "two calls on the same device buffers differ"
    # the same rows through the graph path (one plan image per 1000 bytes)
    from gpuhelp import NativeSession
    with NativeSession(native, plan.blob) as s:
        graph = s.run(x, nbytes // plan.tensors[o.a].bytes)
    rows = sorted(set((np.flatnonzero(got != y_ref) // width).tolist()))
    grows = sorted(set((np.flatnonzero(graph != y_ref) // width).tolist()))
    # the operator call on the library's own device buffers (a session's batch buffers)
    import ctypes as C2
    with NativeSession(native, plan.blob) as s:
        images = nbytes // plan.tensors[o.a].bytes
        din, dout = C2.c_void_p(), C2.c_void_p()
        assert native.ug_batch_buffers(s.handle, images, C2.byref(din), C2.byref(dout)) == 0
        assert native.ug_upload_batch(s.handle, x.ctypes.data, images) == 0
        ops.uq_softmax_exact(din.value, dout.value, nbytes, dq)
        own = np.empty(nbytes, dtype=np.int8)
        assert native.ug_download_batch(s.handle, own.ctypes.data, images) == 0
    orows = sorted(set((np.flatnonzero(own != y_ref) // width).tolist()))
    detail = ""
    for r in rows[:2]:
        sl = slice(r * width, (r + 1) * width)
        detail += (f" | row {r}: x max {int(x[sl].max())}, ours {got[sl][:10].tolist()} ref {y_ref[sl][:10].tolist()}"
                   f" own {own[sl][:10].tolist()}")
    assert not orows, f"on library buffers too: {orows[:12]}{detail}"
    assert not rows and not grows, (f"operator ABI rows differing: {rows[:12]}; graph path rows differing: {grows[:12]}"
                                    f"{detail}")


@pytest.mark.parametrize("name", ["bmm", "bmm_adj", "bmm_attn_qk", "bmm_attn_v", "bmm_odd_k"])
def test_bmm(name, ops, ref, dev):
    plan, o = _op_case(name)
    q = plan.data(o.p[0]).view(np.int32).copy()
    a, b, z = (plan.tensors[t] for t in (o.a, o.b, o.out))
    x, w = seeded(a.bytes, 5), seeded(b.bytes, 6)
    y_ref = np.empty(z.bytes, dtype=np.int8)
    rc_ref = ref.uq_bmm(C.byref(a), C.byref(b), C.byref(z), x.ctypes.data, w.ctypes.data, y_ref.ctypes.data,
                        q.ctypes.data, 1)
    dy = dev.empty(z.bytes)
    rc = ops.uq_bmm(C.byref(a), C.byref(b), C.byref(z), dev.put(x), dev.put(w), dy, dev.put(q), 1)
    assert rc_ref == 0 and rc == 0, (rc_ref, rc, ops.ug_last_error())
    np.testing.assert_array_equal(dev.get(dy, z.bytes), y_ref)


def _gemm_operands(m, n, k, xs, seed):
    rng = np.random.default_rng(seed)
    x = rng.integers(0, 256, size=m * xs, dtype=np.int64).astype(np.uint8)
    w = rng.integers(-128, 128, size=((n + 3) // 4 * 4) * k, dtype=np.int64).astype(np.int8)
    return x, w


SENTINEL = 0x5A5A5A5A


@pytest.mark.parametrize("fn,m,n,k,xs,extra", [
    ("ug_matmul_u8i8", 37, 29, 53, 53, (0, 1)),      # row-major weights, ragged everything
    ("ug_matmul_u8i8", 64, 40, 64, 64, (1, 1)),      # packed
    ("ug_matmul_u8i8", 130, 132, 264, 264, (1, 2)),
    ("ug_matmul_u8i8_strided", 33, 20, 48, 56, ()),
    ("ug_matmul_u8i8_strided", 70, 64, 8192, 8192, ()),
    ("ug_matmul_u8i8_dot4", 34, 12, 40, 48, ()),
    ("ug_matmul_u8i8_dot4", 20, 16, 8, 8, ()),
    ("ug_matmul_u8i8_dot4", 18, 8, 16, 24, ()),
    ("ug_matmul_u8i8_dot4", 66, 36, 32, 32, ()),
    ("ug_matmul_u8i8_dot4", 12, 4, 64, 72, ()),
    ("ug_matmul_u8i8_selected", 9, 32, 64, 64, ()),
    ("ug_matmul_u8i8_selected", 65, 96, 128, 136, ()),
])
def test_gemm_family(fn, m, n, k, xs, extra, ops, ref, dev):
    x, w = _gemm_operands(m, n, k, xs, m * 1000 + k)
    groups = np.array([4, 16, n - 4], dtype=np.uint16) if fn.endswith("selected") else None
    y_ref = np.full(m * n, SENTINEL, dtype=np.int32)

    def args(xp, wp, yp, gp):
        if fn == "ug_matmul_u8i8":
            return (xp, wp, yp, m, n, k) + extra
        if groups is not None:
            return (xp, wp, yp, m, n, k, xs, gp, len(groups))
        return (xp, wp, yp, m, n, k, xs)

    rc_ref = getattr(ref, fn)(*args(x.ctypes.data, w.ctypes.data, y_ref.ctypes.data,
                                    groups.ctypes.data if groups is not None else None))
    dy = dev.empty(m * n * 4, fill=0x5A)
    rc = getattr(ops, fn)(*args(dev.put(x), dev.put(w), dy, groups.ctypes.data if groups is not None else None))
    assert rc_ref == 0 and rc == 0, (rc_ref, rc, ops.ug_last_error())
    np.testing.assert_array_equal(dev.get(dy, m * n * 4, np.int32), y_ref)


def test_gemm_argument_rules_match_reference(ops, ref, dev):
    x, w = _gemm_operands(8, 8, 64, 64, 1)
    dx, dw, dy = dev.put(x), dev.put(w), dev.empty(8 * 8 * 4)
    yh = np.empty(64, dtype=np.int32)
    for fn, a in [("ug_matmul_u8i8_strided", (8, 8, 64, 60)), ("ug_matmul_u8i8_strided", (8, 6, 64, 64)),
                  ("ug_matmul_u8i8_dot4", (7, 8, 64, 64)), ("ug_matmul_u8i8_dot4", (8, 8, 12, 64))]:
        assert getattr(ref, fn)(x.ctypes.data, w.ctypes.data, yh.ctypes.data, *a) == 18
        assert getattr(ops, fn)(dx, dw, dy, *a) == 18
    assert ops.ug_gemm_available() == 1
