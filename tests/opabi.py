"""Helpers for the operator-ABI tests (include/unoq_ops.h): plan parsing into UGTensor / UGOp
records, ctypes bindings of the operator symbols for both libunoq_cuda.so (device buffers) and the
reference build oracle/_ref/libug_ref.so (host buffers: the same symbols of runtime/qnn.c and
runtime/gemm.c)."""
import ctypes as C
import struct

import numpy as np


class UGTensor(C.Structure):
    _fields_ = [("offset", C.c_uint32), ("bytes", C.c_uint32), ("type", C.c_uint32), ("rank", C.c_uint32),
                ("d", C.c_uint32 * 4), ("flags", C.c_uint32), ("reserved", C.c_uint32 * 3)]


class UGOp(C.Structure):
    _fields_ = [("code", C.c_uint32), ("a", C.c_uint32), ("b", C.c_uint32), ("out", C.c_uint32),
                ("p", C.c_uint32 * 4)]


P = C.c_void_p
SIGNATURES = {
    "uq_validate": (C.c_int, [C.POINTER(UGOp)] + [C.POINTER(UGTensor)] * 4 + [P, P, C.POINTER(C.c_uint64)]),
    "uq_run": (C.c_int, [C.c_uint, C.POINTER(UGTensor), C.POINTER(UGTensor), P, P, P, P, C.c_int]),
    "uq_add": (None, [P, P, P, C.c_uint32, P]),
    "uq_mean": (None, [P, P, C.c_uint, C.c_uint, P]),
    "uq_mul": (None, [P, P, P, C.c_uint, P]),
    "uq_bmm": (C.c_int, [C.POINTER(UGTensor)] * 3 + [P, P, P, P, C.c_int]),
    "uq_post_reset": (None, []),
    "uq_post_register": (None, [P, P]),
    "uq_softmax_exact": (None, [P, P, C.c_uint, P]),
    "uq_status": (C.c_int, []),
    "uq_prepare_reset": (None, []),
    "ug_matmul_u8i8": (C.c_int, [P, P, P, C.c_uint, C.c_uint, C.c_uint, C.c_int, C.c_int]),
    "ug_matmul_u8i8_strided": (C.c_int, [P, P, P, C.c_uint, C.c_uint, C.c_uint, C.c_uint]),
    "ug_matmul_u8i8_dot4": (C.c_int, [P, P, P, C.c_uint, C.c_uint, C.c_uint, C.c_uint]),
    "ug_matmul_u8i8_selected": (C.c_int, [P, P, P, C.c_uint, C.c_uint, C.c_uint, C.c_uint, P, C.c_uint]),
    "ug_gemm_available": (C.c_int, []),
}
OP_SYMBOLS = [n for n in SIGNATURES if n not in ("uq_prepare_reset",)]


def bind(lib):
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is not None:
            fn.restype, fn.argtypes = res, args
    return lib


def reference_lib():
    from oracle.oracle import REF_LIB
    if not REF_LIB.is_file():
        return None
    return bind(C.CDLL(str(REF_LIB), mode=C.RTLD_LOCAL))


class Plan:
    """The UGN1 records of a plan (runtime/graph.h:15-38) and views of its constants."""

    def __init__(self, blob):
        self.blob = bytes(blob)
        (self.magic, self.version, self.nt, self.no, self.arena_bytes, self.input, self.output,
         self.reserved) = struct.unpack_from("<8I", self.blob)
        base = 32
        self.tensors = [UGTensor.from_buffer_copy(self.blob, base + 48 * i) for i in range(self.nt)]
        base += 48 * self.nt
        self.ops = [UGOp.from_buffer_copy(self.blob, base + 32 * i) for i in range(self.no)]
        self.arena = np.frombuffer(self.blob, dtype=np.uint8, offset=base + 32 * self.no)

    def data(self, t):
        ts = self.tensors[t]
        return self.arena[ts.offset:ts.offset + ts.bytes].copy()


def batched(t, images):
    """Descriptor `t` with its first axis multiplied by `images` (images back to back)."""
    u = UGTensor.from_buffer_copy(bytes(t))
    u.d[0] = t.d[0] * images
    u.bytes = t.bytes * images
    return u


class Device:
    """Device copies of numpy arrays (torch CUDA tensors kept alive by this object)."""

    def __init__(self):
        import torch
        self.torch = torch
        self.keep = []

    def put(self, a, pad=0):
        """Device copy of `a`; with `pad`, the data starts `pad` bytes into the allocation."""
        a = np.ascontiguousarray(a).reshape(-1).view(np.uint8)
        t = self.torch.zeros(a.nbytes + pad + 1, dtype=self.torch.uint8, device="cuda:0")
        if a.nbytes:
            t[pad:pad + a.nbytes] = self.torch.from_numpy(a.copy()).to("cuda:0")
        self.keep.append(t)
        return t.data_ptr() + pad

    def empty(self, nbytes, pad=0, fill=0x5A):
        t = self.torch.full((nbytes + pad + 1,), fill, dtype=self.torch.uint8, device="cuda:0")
        self.keep.append(t)
        return t.data_ptr() + pad

    def get(self, ptr, nbytes, dtype=np.int8):
        self.torch.cuda.synchronize()
        for t in self.keep:
            lo = t.data_ptr()
            if lo <= ptr and ptr + nbytes <= lo + t.numel():
                return t[ptr - lo:ptr - lo + nbytes].cpu().numpy().view(dtype).copy()
        raise KeyError("pointer not allocated here")
