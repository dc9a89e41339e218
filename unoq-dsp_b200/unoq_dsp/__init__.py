"""unoq_dsp on B200: compiled INT8 vision models executed by CUDA kernels, no CPU fallback.

The public surface follows the reference package (src/unoq_dsp/__init__.py): ``load``,
``CompiledModel``, ``Session``, ``ImageClassifier``, ``ObjectDetector`` and the error types.
``compile_model`` needs the TFLite toolchain of the reference and is not provided here.
"""
from pathlib import Path

from .bundle import CompiledModel, load
from .errors import DSPError, InvalidBundle, UnsupportedModel
from .transport import HardwareSession

__version__ = "0.1.0"


def compile_model(path, *, dsp_threads=2, reuse_memory=True):
    raise UnsupportedModel("TFLite compilation is not part of the CUDA backend; pass a compiled .uqmodel")


class Session(HardwareSession):
    def __init__(self, model, *, library=None, pipeline="rpc"):
        if not isinstance(model, CompiledModel):
            path = Path(model)
            model = load(path) if path.suffix == ".uqmodel" else compile_model(path)
        self._open_plan(model.plan, model.metadata, library, pipeline)


__all__ = ["compile_model", "load", "CompiledModel", "Session", "DSPError", "InvalidBundle", "UnsupportedModel"]

from .vision import ImageClassifier, ObjectDetector  # noqa: E402  (vision imports Session from here)

__all__ += ["ImageClassifier", "ObjectDetector"]
