"""Build libqwen3_b200.so (sm_100a) in-tree with nvcc.

The library is compiled from common_b200/csrc/*.cu into common_b200/lib/libqwen3_b200.so.
Objects are rebuilt only when a source or header is newer than the library.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIBDIR = os.path.join(HERE, "lib")
OBJDIR = os.path.join(LIBDIR, "obj")
LIB = os.path.join(LIBDIR, "libqwen3_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]


def _nccl_link():
    """Link the NCCL that torch itself loads (the nvidia-nccl wheel), so that the library and torch share
    one libnccl.so.2 in a process, whichever is loaded first; the system NCCL otherwise."""
    try:
        import nvidia.nccl
        for base in nvidia.nccl.__path__:
            lib = os.path.join(base, "lib")
            if os.path.exists(os.path.join(lib, "libnccl.so.2")):
                return [f"-L{lib}", "-l:libnccl.so.2", "-Xlinker", f"-rpath,{lib}"]
    except ImportError:
        pass
    return ["-lnccl"]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                  + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, verbose=False):
    obj = os.path.join(OBJDIR, os.path.basename(src) + ".o")
    if not _stale(obj, [src] + _headers()):
        return obj, ""
    cmd = [NVCC] + ARCH + FLAGS + (["-Xptxas", "-v"] if verbose else []) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
    return obj, r.stderr


def build(verbose: bool = False) -> str:
    os.makedirs(OBJDIR, exist_ok=True)
    srcs = _sources()
    # an up-to-date library needs no objects (they are not shipped with a copy of the tree)
    if not verbose and os.path.exists(LIB) and not _stale(LIB, srcs + _headers()):
        return LIB
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), srcs))
    objs = [o for o, _ in results]
    if verbose:
        for _, log in results:
            if log:
                sys.stderr.write(log)
    if _stale(LIB, objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + _nccl_link() + ["-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
