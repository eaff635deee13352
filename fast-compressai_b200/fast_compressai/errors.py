"""Common runtime errors."""


class UnsupportedOperationError(NotImplementedError):
    """Raised when a model path is not available in this build."""
