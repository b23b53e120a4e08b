"""Build the native library ``flashslice_b200/_native/libflashslice_b200.so``.

Compiles every ``csrc/*.cu`` for sm_100a with nvcc and links them into one
shared library exposing the C ABI of ``include/flashslice_b200.h``. The
library is built in-tree so that it travels with the source tree; the
Python package loads it with ctypes and fails loudly when it is missing.

    python -m flashslice_b200.build [--verbose]
"""

import hashlib
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OUTDIR = os.path.join(PKG, "_native")
LIBNAME = "libflashslice_b200.so"
LIBPATH = os.path.join(OUTDIR, LIBNAME)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden"]


def _nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _digest():
    h = hashlib.sha256()
    files = sources() + sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC)
                               if f.endswith((".cuh", ".h")))
    files.append(os.path.join(INCLUDE, "flashslice_b200.h"))
    for f in files:
        with open(f, "rb") as fh:
            h.update(f.encode())
            h.update(fh.read())
    h.update(" ".join(ARCH + FLAGS).encode())
    return h.hexdigest()


def build(verbose=False, force=False):
    """Compile the library unless an up-to-date build is present. Returns the
    library path."""
    os.makedirs(OUTDIR, exist_ok=True)
    stamp = os.path.join(OUTDIR, "build.sha256")
    digest = _digest()
    if not force and os.path.exists(LIBPATH) and os.path.exists(stamp):
        with open(stamp) as f:
            if f.read().strip() == digest:
                return LIBPATH
    objs = []
    for src in sources():
        obj = os.path.join(OUTDIR, os.path.basename(src)[:-3] + ".o")
        cmd = [_nvcc()] + ARCH + FLAGS + ["-I", INCLUDE, "-I", CSRC, "-c",
                                          src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIBPATH + ".tmp"
    cmd = [_nvcc()] + ARCH + ["-shared", "-o", tmp] + objs
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIBPATH)
    for o in objs:
        os.remove(o)
    with open(stamp, "w") as f:
        f.write(digest)
    return LIBPATH


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force="--force" in sys.argv))
