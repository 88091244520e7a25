"""The Node-API addon (ameva-forge_b200/node/forge_b200_addon.cc) compiles
against the C ABI of include/forge_b200.h.  Node.js and its headers are not
installed here, so the check is g++ -fsyntax-only against a declaration stub
of the Node-API subset the addon uses: a changed or removed fg_* signature
fails this test."""
import os
import shutil
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_addon_compiles_against_the_abi():
    r = subprocess.run(["g++", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-fsyntax-only",
                        "-I" + os.path.join(REPO, "tests", "node_api_stub"), "-I" + os.path.join(REPO, "include"),
                        os.path.join(REPO, "ameva-forge_b200", "node", "forge_b200_addon.cc")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_host_module_names_the_reference_surface():
    src = open(os.path.join(REPO, "ameva-forge_b200", "node", "gpuCore.ts")).read()
    # the gpuCore op object (gpuCore.ts:1448-1467) and the bridge object (pyodideBridge.ts:31-58)
    for name in ("add", "mul", "matmul", "matmulTiled", "flashAttention", "rmsNorm", "rope", "swiglu", "unpackQuant",
                 "embedding", "embedding_backward", "adam_step", "sgd_momentum_step", "sparseCrossEntropy",
                 "sparseCrossEntropyBackward", "relu", "relu_backward", "transpose", "init", "read", "dispose",
                 "getTensorInfo", "mapBufferAsync", "readMappedInto", "executeGraph", "warmupKernels", "disposeBatch",
                 "getQuotaSnapshot", "snapshotHandles", "flushGC", "registerPyodideBridge"):
        assert name in src, name
