"""Session over the CUDA backend: the reference's HardwareSession contract, plus batches.

As in the reference (src/unoq_dsp/transport.py:19-85): one active model per process, calls
serialised by a lock, idempotent close, input shape/dtype checked against the manifest, packed
multi-output tensors unpacked (and optionally dequantised) by name. ``run_batch`` is the
extension: it takes (N, *input_shape[1:]) images and returns N stacked results.
"""
import ctypes as C
import threading

import numpy as np

from .errors import DSPError
from .native import last_error, load_library


class HardwareSession:
    """One active session per process; see the module docstring."""

    handle = None

    def _open_plan(self, plan, metadata, library, pipeline):
        if pipeline not in ("mailbox", "rpc"):
            raise ValueError("pipeline must be mailbox or rpc")
        self.metadata = metadata
        self.lock = threading.Lock()
        self.handle = None
        self.lib = load_library(library)
        error = C.c_int()
        self._plan = C.create_string_buffer(bytes(plan), len(plan))
        handle = self.lib.ug_open_mode(self._plan, len(plan), int(pipeline == "mailbox"), C.byref(error))
        if not handle:
            code = error.value & 0xFFFFFFFF
            raise DSPError(f"Model load failed: {code:#010x} {last_error(self.lib)}; no CPU fallback".rstrip())
        self.handle = handle

    def _unpack(self, y):
        if not self.metadata.get("outputs"):
            return y
        wire = y.reshape(-1).view("u1")
        result = {}
        for spec in self.metadata["outputs"]:
            lo = spec["packed_offset"]
            value = wire[lo:lo + spec["bytes"]].view(spec["dtype"]).reshape(spec["shape"])
            if spec.get("dequantize"):
                q = spec["quantization"]
                value = (value.astype("f4") - np.float32(q["zero_point"])) * np.float32(q["scale"])
            result[spec["name"]] = value
        return next(iter(result.values())) if len(result) == 1 else result

    def run(self, x):
        with self.lock:
            if not self.handle:
                raise DSPError("Session closed")
            spec = self.metadata["input"]
            x = np.asarray(x)
            if x.shape != tuple(spec["shape"]) or x.dtype != np.dtype(spec["dtype"]):
                raise ValueError(f"Expected {tuple(spec['shape'])} {spec['dtype']}")
            x = np.ascontiguousarray(x)
            out = self.metadata["output"]
            y = np.empty(out["shape"], dtype=out["dtype"])
            rc = self.lib.ug_infer(self.handle, x.ctypes.data, x.nbytes, y.ctypes.data, y.nbytes)
            if rc:
                raise DSPError(f"Inference failed: {rc & 0xFFFFFFFF:#010x} {last_error(self.lib)}; no CPU fallback")
            return self._unpack(y)

    def run_batch(self, x):
        """Run N images at once: x has shape (N, *input_shape[1:]); returns a list of N results
        (each as ``run`` would return it) when the model has packed outputs, else an array."""
        with self.lock:
            if not self.handle:
                raise DSPError("Session closed")
            spec = self.metadata["input"]
            x = np.ascontiguousarray(np.asarray(x))
            per = tuple(spec["shape"])
            if x.ndim != len(per) or x.shape[1:] != per[1:] or x.dtype != np.dtype(spec["dtype"]) or per[0] != 1:
                raise ValueError(f"Expected (N, {', '.join(map(str, per[1:]))}) {spec['dtype']}")
            n = x.shape[0]
            out = self.metadata["output"]
            y = np.empty((n,) + tuple(out["shape"]), dtype=out["dtype"])
            rc = self.lib.ug_infer_batch(self.handle, x.ctypes.data, n, y.ctypes.data)
            if rc:
                raise DSPError(f"Batch inference failed: {rc & 0xFFFFFFFF:#010x} {last_error(self.lib)}")
            if self.metadata.get("outputs"):
                return [self._unpack(y[i]) for i in range(n)]
            return y

    def close(self):
        lock = getattr(self, "lock", None)
        if lock is None:
            return
        with lock:
            if self.handle:
                self.lib.ug_close(self.handle)
                self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *args):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
