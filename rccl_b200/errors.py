"""Python mirror of rccl_cub::DeviceAlgorithmError (rccl-cub/src/error.rs:1-84).

Each C status code (include/rsort_b200.h) maps to one exception class whose
payload matches the Rust variant's fields.
"""
from __future__ import annotations

from . import _lib


class DeviceAlgorithmError(Exception):
    """Failure reported by a device-wide operation (error.rs:3)."""


class LengthMismatch(DeviceAlgorithmError):
    def __init__(self, role: str, expected: int, actual: int):
        self.role, self.expected, self.actual = role, expected, actual
        super().__init__(f"{role} length {actual} does not match required length {expected}")


class WorkspaceTooSmall(DeviceAlgorithmError):
    def __init__(self, role: str, required: int, actual: int):
        self.role, self.required, self.actual = role, required, actual
        super().__init__(f"{role} length {actual} is smaller than required length {required}")


class InvalidBitRange(DeviceAlgorithmError):
    def __init__(self, begin: int, end: int, key_bits: int):
        self.begin, self.end, self.key_bits = begin, end, key_bits
        super().__init__(f"radix bit range {begin}..{end} is outside 0..={key_bits} or reversed")


class UnsupportedTarget(DeviceAlgorithmError):
    pass


class SizeOverflow(DeviceAlgorithmError):
    def __init__(self, message: str = "combined device range length overflowed"):
        super().__init__(message)


class DriverError(DeviceAlgorithmError):
    """CUDA driver or launch failure (the Driver / Launch variants)."""


class DeviceTimeout(DeviceAlgorithmError):
    """A bounded device wait gave up (no reference variant: its waits are unbounded)."""


class BadArgument(DeviceAlgorithmError):
    """Unsupported layout or malformed argument (the reference rejects these statically)."""


def raise_for(status: int) -> None:
    """Raise the exception matching a non-OK rsort_status."""
    if status == _lib.RSORT_OK:
        return
    info = _lib.last_error()
    role = info.role.decode() if info.role else ""
    if status == _lib.RSORT_INVALID_BIT_RANGE:
        raise InvalidBitRange(info.begin_bit, info.end_bit, info.key_bits)
    if status == _lib.RSORT_LENGTH_MISMATCH:
        raise LengthMismatch(role, info.expected, info.actual)
    if status == _lib.RSORT_WORKSPACE_TOO_SMALL:
        raise WorkspaceTooSmall(role, info.expected, info.actual)
    if status == _lib.RSORT_UNSUPPORTED_TARGET:
        raise UnsupportedTarget(role)
    if status == _lib.RSORT_SIZE_OVERFLOW:
        raise SizeOverflow(role or "combined device range length overflowed")
    if status == _lib.RSORT_TIMEOUT:
        raise DeviceTimeout(role)
    if status == _lib.RSORT_CUDA_ERROR:
        raise DriverError(role)
    raise BadArgument(role or f"status {status}")
