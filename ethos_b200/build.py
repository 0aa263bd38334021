"""Build the sm_100a shared library ``ethos_b200/libethos_b200.so`` in tree.

    python -m ethos_b200.build          # or: from ethos_b200.build import build; build()

nvcc cross-compiles for sm_100a without a GPU, so this runs on any host with
CUDA 12.9.  The library is rebuilt when a source or header is newer than it.
"""

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB_NAME = "libethos_b200.so"
LIB_PATH = os.path.join(PKG, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path():
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _sources():
    srcs, deps = [], []
    for name in sorted(os.listdir(CSRC)):
        p = os.path.join(CSRC, name)
        if name.endswith(".cu"):
            srcs.append(p)
        if name.endswith((".cu", ".cuh", ".h")):
            deps.append(p)
    for name in sorted(os.listdir(INCLUDE)):
        deps.append(os.path.join(INCLUDE, name))
    return srcs, deps


def needs_build(out=LIB_PATH):
    if not os.path.exists(out):
        return True
    mtime = os.path.getmtime(out)
    _, deps = _sources()
    return any(os.path.getmtime(d) > mtime for d in deps)


def build(force=False, verbose=False, extra_flags=()):
    """Compile every ``csrc/*.cu`` into one shared library (sm_100a only)."""
    if not force and not needs_build():
        return LIB_PATH
    srcs, _ = _sources()
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "--shared",
           "-Xcompiler", "-fPIC,-O3", "-I", INCLUDE, "-I", CSRC,
           "--expt-relaxed-constexpr", *extra_flags, "-o", tmp, *srcs]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building %s" % LIB_NAME)
    if verbose and (res.stdout or res.stderr):
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    force = "--force" in sys.argv
    verbose = "-v" in sys.argv or "--verbose" in sys.argv
    extra = ["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else []
    print(build(force=force, verbose=verbose or bool(extra), extra_flags=extra))
