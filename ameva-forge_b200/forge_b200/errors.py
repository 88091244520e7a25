"""Typed errors of the forge_b200 host API.

One class per typed error of the reference (packages/forge/src/errors.ts:
12-111), with the same names, so code that catches the reference's errors by
name (forge-py bridge.py:206-226 maps JS error names to exceptions) keeps
working.  The C ABI returns the matching status code; ``raise_for`` turns it
into the exception carrying the library's message.
"""


class AMEVAForgeError(Exception):
    status = -1


class AMEVAForgeShapeError(AMEVAForgeError):
    status = 1


class AMEVAForgeDTypeError(AMEVAForgeError):
    status = 2


class AMEVAForgeDeviceError(AMEVAForgeError):
    status = 3


class AMEVAForgeDisposedError(AMEVAForgeError):
    status = 4


class AMEVAForgeQuotaExceededError(AMEVAForgeError):
    status = 5


class AMEVAForgeWebGPUUnavailableError(AMEVAForgeError):
    """No usable accelerator (the reference's name is kept for drop-in use)."""
    status = 6


class AMEVAForgeSecurityError(AMEVAForgeError):
    status = 7


class AMEVAForgeUnsupportedOpError(AMEVAForgeError):
    status = 8


class AMEVAForgeValidationError(AMEVAForgeError):
    status = 9


class AMEVAForgeOutOfMemoryError(AMEVAForgeError):
    status = 10


class AMEVAForgeInternalGPUError(AMEVAForgeError):
    status = 11


class AMEVAForgeDeviceLostError(AMEVAForgeError):
    status = 12


class AMEVAForgeStaleHandleError(AMEVAForgeError):
    status = 13


BY_STATUS = {c.status: c for c in (
    AMEVAForgeShapeError, AMEVAForgeDTypeError, AMEVAForgeDeviceError, AMEVAForgeDisposedError,
    AMEVAForgeQuotaExceededError, AMEVAForgeWebGPUUnavailableError, AMEVAForgeSecurityError,
    AMEVAForgeUnsupportedOpError, AMEVAForgeValidationError, AMEVAForgeOutOfMemoryError,
    AMEVAForgeInternalGPUError, AMEVAForgeDeviceLostError, AMEVAForgeStaleHandleError)}


def raise_for(status: int, message: str):
    if status == 0:
        return
    raise BY_STATUS.get(status, AMEVAForgeError)(message)
