"""Error hierarchy of the AVQ-attention API.

Same class names, constructor signatures and ``context`` dict as the
reference (``src/avqa/exceptions.py:11-179``), so code that catches the
reference's errors catches these.  A non-zero status from the CUDA C-ABI
surfaces as :class:`BackendError` carrying the library's last error string.
"""
from __future__ import annotations


class AVQAError(Exception):
    """Base class of every error raised by this package."""

    def __init__(self, message: str, context: dict[str, object] | None = None) -> None:
        super().__init__(message)
        self.message = message
        self.context: dict[str, object] = dict(context) if context else {}

    def __str__(self) -> str:
        return f"{self.message} | context={self.context}" if self.context else self.message

    def __repr__(self) -> str:
        return f"{type(self).__name__}({self.message!r}, context={self.context!r})"


class ConfigurationError(AVQAError):
    """Invalid or inconsistent configuration."""


class BackendError(AVQAError):
    """A backend call failed (unknown backend, missing CUDA library, kernel error)."""


class RoutingError(AVQAError):
    """Routing cannot produce a decision (bad budget, bad importance shape)."""


class CodebookError(AVQAError):
    """Codebook construction or update failed."""


class MergeError(AVQAError):
    """A merge strategy failed."""


class _ExpectedActual(AVQAError):
    def __init__(self, message: str, expected: object = None, actual: object = None,
                 context: dict[str, object] | None = None) -> None:
        merged: dict[str, object] = dict(context) if context else {}
        if expected is not None:
            merged["expected"] = expected
        if actual is not None:
            merged["actual"] = actual
        super().__init__(message, merged)


class ShapeError(_ExpectedActual):
    """A tensor shape violates the documented contract."""


class DtypeError(_ExpectedActual):
    """A tensor dtype is unsupported or mismatched."""


class DeviceError(_ExpectedActual):
    """A tensor lives on an unsupported or mismatched device."""


class NotInitializedError(AVQAError):
    """A required component has not been initialised."""


__all__ = [
    "AVQAError", "BackendError", "CodebookError", "ConfigurationError", "DeviceError", "DtypeError",
    "MergeError", "NotInitializedError", "RoutingError", "ShapeError",
]
