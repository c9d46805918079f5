"""Builds librazorkv_b200.so (the C-ABI CUDA library) in-tree for sm_100a.

    python -m razorkv_b200.build            # incremental
    python -m razorkv_b200.build --force    # rebuild every object

nvcc cross-compiles without a GPU.  Objects go to razorkv_b200/_build/, the shared library
to razorkv_b200/_lib/librazorkv_b200.so (both outside version control; the library is
loaded from there at import time).
"""

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ_DIR = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(HERE, "_lib")
LIB_PATH = os.path.join(LIB_DIR, "librazorkv_b200.so")

SOURCES = ["rkv_capi.cu", "rkv_generic.cu", "rkv_decode_sm100.cu", "rkv_noalloc.cu"]
HEADERS = ["rkv_common.cuh", "rkv_kernels.h", "rkv_sm100.cuh"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr", "-Xptxas", "-v",
]


def _nvcc():
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.exists(d) and os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJ_DIR, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    header_paths = [os.path.join(CSRC, h) for h in HEADERS] + [
        os.path.join(ROOT, "include", "razorkv_b200.h")]
    objs = []
    for src in SOURCES:
        sp = os.path.join(CSRC, src)
        op = os.path.join(OBJ_DIR, src.replace(".cu", ".o"))
        objs.append(op)
        if force or _stale(op, [sp] + header_paths + [__file__]):
            cmd = [_nvcc(), *NVCC_FLAGS, "-c", sp, "-o", op]
            res = subprocess.run(cmd, capture_output=True, text=True)
            log = os.path.join(OBJ_DIR, src.replace(".cu", ".ptxas.txt"))
            with open(log, "w") as f:
                f.write(res.stdout + res.stderr)
            if res.returncode != 0:
                sys.stderr.write(res.stdout + res.stderr)
                raise RuntimeError(f"nvcc failed for {src}")
            if verbose:
                sys.stdout.write(res.stderr)
    if force or _stale(LIB_PATH, objs):
        cmd = [_nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", LIB_PATH,
               *objs]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("link of librazorkv_b200.so failed")
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
