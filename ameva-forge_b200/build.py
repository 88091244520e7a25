"""Build libforge_b200.so (sm_100a) in-tree.

    python ameva-forge_b200/build.py [--clean]

Compiles every csrc/*.cu with nvcc for sm_100a only (-gencode
arch=compute_100a,code=sm_100a), links them with NCCL into
forge_b200/_lib/libforge_b200.so and exports only the fg_* C ABI
(include/forge_b200.h).  nvcc cross-compiles, so this runs on a machine
without a GPU; the .so travels with the source tree.
"""
import concurrent.futures
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "forge_b200", "_lib")
LIB = os.path.join(LIBDIR, "libforge_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
                 "-Xcompiler", "-Wno-unused-function", "-I" + os.path.join(HERE, "..", "include")]
EXPORTS = os.path.join(OBJ, "exports.map")


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _needs(obj, src):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    deps = [src] + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".cuh", ".h"))]
    deps.append(os.path.join(HERE, "..", "include", "forge_b200.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src):
    obj = os.path.join(OBJ, src.replace(".cu", ".o"))
    path = os.path.join(CSRC, src)
    if not _needs(obj, path):
        return obj, None
    cmd = [NVCC] + CFLAGS + ["-c", path, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, r.stderr + r.stdout
    return obj, None


def build(verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    with open(EXPORTS, "w") as f:
        f.write("{\n  global: fg_*;\n  local: *;\n};\n")
    srcs = _sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(_compile, srcs))
    errs = [e for _, e in results if e]
    if errs:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errs))
    objs = [o for o, _ in results]
    if not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + [
            "-ldl", "-Xlinker", "--version-script=" + EXPORTS, "-Xlinker", "-z,defs"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stderr + r.stdout)
    if verbose:
        print("built", LIB)
    return LIB


if __name__ == "__main__":
    if "--clean" in sys.argv:
        shutil.rmtree(OBJ, ignore_errors=True)
        if os.path.exists(LIB):
            os.remove(LIB)
    build(verbose=True)
