"""Errors raised by coder backends and payload validation.

Same hierarchy as the reference (coders/errors.py:4-21) so callers can catch
the same types.
"""


class CoderError(RuntimeError):
    """Base class for coder failures."""


class CoderInputError(CoderError, ValueError):
    """Raised when symbols, indexes, CDF metadata or a payload is invalid."""


class CoderStateError(CoderError):
    """Raised when a coder is used in an invalid state."""


class BitstreamError(CoderError, ValueError):
    """Raised for malformed or incompatible bitstreams."""


class CoderDependencyError(CoderError, ImportError):
    """Raised when a coder's native dependency is unavailable."""
