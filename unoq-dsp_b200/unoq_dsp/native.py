"""Locate and bind libunoq_cuda.so (the C ABI of include/unoq_cuda.h) with ctypes.

Library resolution: an explicit path, else ``UNOQ_DSP_LIBRARY`` (the variable the reference's
transport reads, src/unoq_dsp/transport.py:25-30), else the in-tree build at
``unoq-dsp_b200/lib/libunoq_cuda.so``. There is no CPU fallback: a missing library is an error.
"""
import ctypes as C
import os
from pathlib import Path

import numpy as np

from .errors import DSPError

YOLO_MAX_LEVELS = 4


class UgYoloLevel(C.Structure):
    """include/unoq_cuda.h UgYoloLevel."""
    _fields_ = [("box_offset", C.c_uint32), ("score_offset", C.c_uint32), ("height", C.c_uint32),
                ("width", C.c_uint32), ("stride", C.c_float), ("distance", C.c_float * 256),
                ("score", C.c_float * 256), ("rank", C.c_uint16 * 256)]


class UgYoloDecode(C.Structure):
    """include/unoq_cuda.h UgYoloDecode."""
    _fields_ = [("levels", C.c_uint32), ("classes", C.c_uint32), ("candidates", C.c_uint32),
                ("reserved", C.c_uint32), ("level", UgYoloLevel * YOLO_MAX_LEVELS)]


# include/unoq_cuda.h UgDetectionRecord (32 bytes); anchor 0xFFFFFFFF marks "no pair"
RECORD_DTYPE = np.dtype([("anchor", "<u4"), ("class_id", "<u4"), ("score", "<f4"), ("box", "<f4", (4,)),
                         ("reserved", "<u4")])
NO_ANCHOR = 0xFFFFFFFF

DEFAULT_LIBRARY = Path(__file__).resolve().parents[1] / "lib" / "libunoq_cuda.so"

_SIGNATURES = {
    "ug_load": (C.c_int, [C.c_void_p, C.c_uint32]),
    "ug_run": (C.c_int, [C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32]),
    "ug_input_bytes": (C.c_uint32, []),
    "ug_output_bytes": (C.c_uint32, []),
    "ug_snapshot": (C.c_int, [C.c_uint32, C.c_void_p, C.c_uint32]),
    "ug_profile": (C.c_int, [C.c_uint32, C.c_void_p, C.c_uint32]),
    "ug_open_mode": (C.c_void_p, [C.c_void_p, C.c_uint32, C.c_int, C.POINTER(C.c_int)]),
    "ug_open": (C.c_void_p, [C.c_void_p, C.c_uint32, C.POINTER(C.c_int)]),
    "ug_infer": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32]),
    "ug_close": (None, [C.c_void_p]),
    "ug_snapshot_tensor": (C.c_int, [C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32]),
    "ug_profile_control": (C.c_int, [C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32]),
    "ug_set_device": (C.c_int, [C.c_int]),
    "ug_infer_batch": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_void_p]),
    "ug_batch_buffers": (C.c_int, [C.c_void_p, C.c_uint32, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)]),
    "ug_launch_batch": (C.c_int, [C.c_void_p, C.c_uint32]),
    "ug_synchronize": (C.c_int, [C.c_void_p]),
    "ug_time_batch": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.POINTER(C.c_float)]),
    "ug_last_infer_ms": (C.c_float, [C.c_void_p]),
    "ug_host_alloc": (C.c_void_p, [C.c_size_t]),
    "ug_host_free": (None, [C.c_void_p]),
    "ug_validate_plan": (C.c_int, [C.c_void_p, C.c_uint32]),
    "ug_batch_kernel_count": (C.c_int, [C.c_void_p, C.c_uint32]),
    "ug_run_static": (C.c_int, [C.c_void_p, C.c_uint32, C.c_void_p, C.c_uint32]),
    "ug_upload_batch": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32]),
    "ug_download_batch": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32]),
    "ug_dist_unique_id": (C.c_int, [C.c_void_p, C.c_uint32]),
    "ug_dist_init": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_uint32]),
    "ug_gather_buffer": (C.c_int, [C.c_void_p, C.c_uint32, C.POINTER(C.c_void_p)]),
    "ug_time_gather": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.POINTER(C.c_float)]),
    "ug_profile_batch": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.POINTER(C.c_uint64), C.c_uint32,
                                   C.POINTER(C.c_float)]),
    "ug_set_input_table": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32]),
    "ug_set_yolo_decode": (C.c_int, [C.c_void_p, C.POINTER(UgYoloDecode)]),
    "ug_detect_batch": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p]),
    "ug_launch_detect": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32]),
    "ug_detect_buffer": (C.c_int, [C.c_void_p, C.c_uint32, C.c_uint32, C.POINTER(C.c_void_p)]),
    "ug_measure_int8_peak": (C.c_int, [C.c_uint32, C.POINTER(C.c_float), C.POINTER(C.c_float)]),
    "ug_last_error": (C.c_char_p, []),
}

_cache = {}


def library_path(explicit=None):
    return Path(explicit or os.environ.get("UNOQ_DSP_LIBRARY") or DEFAULT_LIBRARY)


def load_library(explicit=None):
    path = library_path(explicit).resolve()
    if path in _cache:
        return _cache[path]
    if not path.is_file():
        raise DSPError(f"CUDA backend library not found at {path}; build it with unoq-dsp_b200/build.py")
    try:
        lib = C.CDLL(str(path))
    except OSError as exc:
        raise DSPError(f"Cannot load CUDA backend library: {exc}") from exc
    for name, (restype, argtypes) in _SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = restype
        fn.argtypes = argtypes
    _cache[path] = lib
    return lib


def last_error(lib):
    msg = lib.ug_last_error() if hasattr(lib, "ug_last_error") else b""
    return msg.decode(errors="replace") if msg else ""
