"""Build the sm_100a shared library ``libcirrus_b200.so`` in-tree with nvcc.

    python -m cirrus_s_1a_b200.build        # or: from cirrus_s_1a_b200.build import build; build()

Every ``csrc/*.cu`` is compiled for ``arch=compute_100a,code=sm_100a`` and
linked into one position-independent shared library next to this file; the
library exports the C ABI declared in ``include/cirrus_b200.h``.  An object is
recompiled only when its source or a header is newer than it; objects compile
in parallel.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libcirrus_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def sources() -> list:
    return sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")))


def _headers() -> list:
    return glob.glob(os.path.join(HERE, "csrc", "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def _newer(target: str, deps: list) -> bool:
    """True when ``target`` is missing or older than any of ``deps``."""
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(f) > t for f in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    objdir = os.path.join(ROOT, "_build")
    objs = [os.path.join(objdir, os.path.basename(s)[:-3] + ".o") for s in sources()]
    stale = [(s, o) for s, o in zip(sources(), objs) if force or _newer(o, [s, *_headers()])]
    if not stale and not _newer(LIB, objs):
        return LIB
    nvcc = _nvcc()
    os.makedirs(objdir, exist_ok=True)

    def compile_one(pair):
        src, obj = pair
        cmd = [nvcc, *ARCH, *FLAGS, "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)

    with ThreadPoolExecutor(max_workers=max(1, min(len(stale), os.cpu_count() or 1))) as ex:
        list(ex.map(compile_one, stale))
    tmp = LIB + ".tmp"
    subprocess.run([nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", tmp, "-lcudart"], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
