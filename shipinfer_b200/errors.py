"""Error types of the image-ops seam.

The names and meanings follow the reference's ``shipinfer.core.errors`` as the seam uses them
(``src/shipinfer/runtime/ops/native_ops.py:10,22-72,96-127``): a caller that catches the
reference's exceptions around ``ImageOps`` calls catches these by the same names. When the
reference package is importable, these classes derive from its own, so an ``except`` written
against either hierarchy matches.
"""

from __future__ import annotations

try:  # pragma: no cover - depends on whether the reference package is installed
    from shipinfer.core.errors import ConfigurationError as _RefConfigurationError
    from shipinfer.core.errors import ValidationError as _RefValidationError
except Exception:  # the reference is not installed: plain bases
    _RefConfigurationError = Exception  # type: ignore[misc,assignment]
    _RefValidationError = ValueError  # type: ignore[misc,assignment]

__all__ = ["ConfigurationError", "NativeError", "ValidationError"]


class ValidationError(_RefValidationError):  # type: ignore[valid-type,misc]
    """An argument violates the contract (shape, dtype, device, layout)."""


class ConfigurationError(_RefConfigurationError):  # type: ignore[valid-type,misc]
    """The native library is missing, unusable, or was asked for something it cannot do."""


class NativeError(RuntimeError):
    """A CUDA call inside the library failed; the message is the library's own."""
