"""C-ABI checks that need no GPU: the library loads, exports every function
include/forge_b200.h declares, names its statuses after the reference's
error classes, and fails loudly (no CPU fallback) when no device exists."""
import ctypes
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "forge_b200.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(fg_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    import forge_b200
    return forge_b200.lib()


def test_header_declares_the_boundary():
    fns = header_functions()
    for required in ("fg_init", "fg_upload_quant", "fg_unpack_quant", "fg_qmatmul", "fg_flash_attention",
                     "fg_llama_decode", "fg_last_error"):
        assert required in fns


def test_library_exports_every_declared_symbol(lib):
    missing = [f for f in header_functions() if not hasattr(lib, f)]
    assert not missing, missing


def test_library_exports_nothing_else():
    import subprocess
    import forge_b200
    out = subprocess.run(["nm", "-D", "--defined-only", forge_b200.LIB_PATH], capture_output=True, text=True).stdout
    syms = {l.split()[-1] for l in out.splitlines() if " T " in l}
    assert syms == set(header_functions()), syms ^ set(header_functions())


def test_status_names_follow_reference_error_classes(lib):
    from forge_b200 import errors
    names = {s: lib.fg_status_name(s).decode() for s in range(1, 14)}
    for s, cls in errors.BY_STATUS.items():
        assert names[s] == cls.__name__
    # the reference's class list (packages/forge/src/errors.ts:32-111)
    assert sorted(names.values()) == sorted([
        "AMEVAForgeShapeError", "AMEVAForgeDTypeError", "AMEVAForgeDeviceError", "AMEVAForgeDisposedError",
        "AMEVAForgeQuotaExceededError", "AMEVAForgeWebGPUUnavailableError", "AMEVAForgeSecurityError",
        "AMEVAForgeUnsupportedOpError", "AMEVAForgeValidationError", "AMEVAForgeOutOfMemoryError",
        "AMEVAForgeInternalGPUError", "AMEVAForgeDeviceLostError", "AMEVAForgeStaleHandleError"])


def test_version(lib):
    assert b"sm_100a" in lib.fg_version()


def test_init_without_device_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import forge_b200
    from forge_b200.errors import AMEVAForgeWebGPUUnavailableError
    with pytest.raises(AMEVAForgeWebGPUUnavailableError):
        forge_b200.Context()
    assert forge_b200.device_count() == 0


def test_bad_handle_is_a_disposed_error():
    from forge_b200.gpu_core import _h
    from forge_b200.errors import AMEVAForgeDisposedError
    with pytest.raises(AMEVAForgeDisposedError):
        _h("not-a-handle")
    assert _h("tensor_00000000000000ff") == 255


def test_null_context_is_a_validation_error(lib):
    h = ctypes.c_uint64()
    st = lib.fg_upload(None, None, 0, None, 0, 0, ctypes.byref(h))
    assert lib.fg_status_name(st).decode() == "AMEVAForgeValidationError"
