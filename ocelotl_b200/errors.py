"""Error types of the quantized-linear backend.

Mirrors the reference's error contract (crates/core/src/lib.rs:14-30 for the
enum, :75-80 for KernelError, :55-64 for UnsupportedError, :48-52 for
InvalidRequestError): a kernel failure carries the backend id and a message;
an unsupported type/shape names the feature, what was requested and what is
supported, and is raised before any launch.
"""
from __future__ import annotations


class OcelotlError(Exception):
    """Base of all errors (OcelotlError)."""


class KernelError(OcelotlError):
    """OcelotlError::Kernel(KernelError{backend, message})."""

    def __init__(self, backend: str, message: str):
        self.backend = backend
        self.message = message
        super().__init__(f"kernel error on backend `{backend}`: {message}")


class UnsupportedError(OcelotlError):
    """OcelotlError::Unsupported(UnsupportedError{feature, requested, supported})."""

    def __init__(self, feature: str, requested: str | None = None, supported: list[str] | None = None,
                 message: str | None = None):
        self.feature = feature
        self.requested = requested
        self.supported = list(supported or [])
        if message is None:
            req = f" (requested `{requested}`)" if requested is not None else ""
            message = f"unsupported feature `{feature}`{req}: supported = [{', '.join(self.supported)}]"
        super().__init__(message)


class InvalidRequestError(OcelotlError):
    """OcelotlError::InvalidRequest(InvalidRequestError{field, message})."""

    def __init__(self, field: str, message: str):
        self.field = field
        self.message = message
        super().__init__(f"invalid request field `{field}`: {message}")
