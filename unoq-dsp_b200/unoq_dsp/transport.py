"""Session over the CUDA backend: the reference's HardwareSession contract, plus batches.

As in the reference (src/unoq_dsp/transport.py:19-85): one active model per process, calls
serialised by a lock, idempotent close, input shape/dtype checked against the manifest, packed
multi-output tensors unpacked (and optionally dequantised) by name. Extensions: ``run_batch``
takes (N, *input_shape[1:]) images and returns N stacked results; ``set_input_table`` moves the
image APIs' byte table onto the GPU (inputs are then uint8 pixels); ``set_yolo_decode`` and
``detect_batch`` run the one-to-one YOLO top-k on the GPU and return its records.
"""
import ctypes as C
import threading

import numpy as np

from .errors import DSPError
from .native import RECORD_DTYPE, last_error, load_library


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
        self.input_table = None
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

    def _input_dtype(self):
        return np.dtype(np.uint8) if self.input_table is not None else np.dtype(self.metadata["input"]["dtype"])

    def _batch_input(self, x):
        spec = self.metadata["input"]
        x = np.ascontiguousarray(np.asarray(x))
        per = tuple(spec["shape"])
        if x.ndim != len(per) or x.shape[1:] != per[1:] or x.dtype != self._input_dtype() or per[0] != 1:
            raise ValueError(f"Expected (N, {', '.join(map(str, per[1:]))}) {self._input_dtype()}")
        return x

    def _check(self, rc, what):
        if rc:
            raise DSPError(f"{what} failed: {rc & 0xFFFFFFFF:#010x} {last_error(self.lib)}; no CPU fallback".rstrip())

    def set_input_table(self, table):
        """Map every input through `table` ((256, channels) int8: byte b of channel c becomes
        table[b, c]) on the GPU; inputs are then uint8 pixels of the input shape. None removes it."""
        with self.lock:
            if not self.handle:
                raise DSPError("Session closed")
            if table is None:
                self._check(self.lib.ug_set_input_table(self.handle, None, 0), "Input table")
                self.input_table = None
                return
            t = np.ascontiguousarray(np.asarray(table))
            if t.ndim != 2 or t.shape[0] != 256 or t.dtype != np.int8:
                raise ValueError("Expected a (256, channels) int8 table")
            self._check(self.lib.ug_set_input_table(self.handle, t.ctypes.data, t.shape[1]), "Input table")
            self.input_table = t

    def set_yolo_decode(self, config):
        """Install the GPU decoder (a native.UgYoloDecode, see YOLODecoder.device_config); None removes it."""
        with self.lock:
            if not self.handle:
                raise DSPError("Session closed")
            self._check(self.lib.ug_set_yolo_decode(self.handle, None if config is None else C.byref(config)),
                        "Decoder set-up")

    def detect_batch(self, x, k):
        """(N, *input_shape[1:]) inputs -> (N, k) RECORD_DTYPE records of the GPU decoder."""
        with self.lock:
            if not self.handle:
                raise DSPError("Session closed")
            x = self._batch_input(x)
            records = np.empty((x.shape[0], k), dtype=RECORD_DTYPE)
            self._check(self.lib.ug_detect_batch(self.handle, x.ctypes.data, x.shape[0], k, records.ctypes.data),
                        "Detection")
            return records

    def run(self, x):
        with self.lock:
            if not self.handle:
                raise DSPError("Session closed")
            spec = self.metadata["input"]
            x = np.asarray(x)
            if x.shape != tuple(spec["shape"]) or x.dtype != self._input_dtype():
                raise ValueError(f"Expected {tuple(spec['shape'])} {self._input_dtype()}")
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
            x = self._batch_input(x)
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
