"""Build libisaac_net_b200.so in-tree with nvcc for sm_100a (B200).

    python isaac-net_b200/build.py            # or __graft_entry__.build()

Each .cu file under csrc/ is compiled to an object in parallel (-gencode arch=compute_100a,code=sm_100a, -O3,
-lineinfo, IEEE division / square root, no fast math), then linked into _lib/libisaac_net_b200.so.  The library is
rebuilt only when a source or header is newer than it.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OUT_DIR = os.path.join(HERE, "_lib")
LIB = os.path.join(OUT_DIR, "libisaac_net_b200.so")
LIB_CHECK = os.path.join(OUT_DIR, "libisaac_net_b200_check.so")   # -DINB_CHECK: bounds-checked debug build
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
              "-prec-div=true", "-prec-sqrt=true", "-ftz=false", f"-I{INCLUDE}", f"-I{CSRC}"]


def _nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.isabs(c) and os.path.exists(c) or not os.path.isabs(c)):
            return c
    return "nvcc"


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale(lib=LIB):
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force=False, verbose=False, extra_flags=(), check=False):
    """Compile and link the library (check=True: the bounds-checked debug variant); returns its path."""
    lib = LIB_CHECK if check else LIB
    if check:
        extra_flags = tuple(extra_flags) + ("-DINB_CHECK",)
    if not force and not _stale(lib):
        return lib
    os.makedirs(OUT_DIR, exist_ok=True)
    nvcc = _nvcc()
    objs = []

    def one(src):
        obj = os.path.join(OUT_DIR, os.path.basename(src)[:-3] + (".chk.o" if check else ".o"))
        cmd = [nvcc, *NVCC_FLAGS, *extra_flags, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        if verbose:
            sys.stderr.write(r.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as ex:
        objs = list(ex.map(one, sources()))
    tmp = lib + ".tmp"
    r = subprocess.run([nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", tmp, *objs],
                       capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, lib)
    for o in objs:
        os.remove(o)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv,
                extra_flags=("-Xptxas", "-v") if "-v" in sys.argv else (), check="--check" in sys.argv))
