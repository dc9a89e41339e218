"""Exceptions of the public API (names and bases as in the reference's src/unoq_dsp/errors.py)."""


class UnsupportedModel(ValueError):
    """The model cannot run under this backend's plan contract."""


class InvalidBundle(ValueError):
    """A compiled .uqmodel is malformed, incompatible or corrupt."""


class DSPError(RuntimeError):
    """Accelerator execution failed. Nothing is silently re-run on the CPU."""
