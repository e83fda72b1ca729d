"""Build ``liblaguna_b200.so`` (the C-ABI library) from ``csrc/*.cu`` for sm_100a, in-tree.

    python -m lagunalab_b200.build

Each ``.cu`` is compiled to an object under ``_build/`` in parallel, then linked with the
static CUDA runtime into ``lagunalab_b200/liblaguna_b200.so``. Objects are rebuilt when the
source or any header is newer.
"""
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "liblaguna_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", str(ROOT / "include")]


def nvcc():
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def _headers():
    return list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))


def _compile(src, verbose=False):
    obj = BUILD / (src.stem + ".o")
    newest = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if obj.exists() and obj.stat().st_mtime >= newest:
        return obj, ""
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(verbose=False):
    """Compile every kernel source and link the shared library. Returns its path."""
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with ThreadPoolExecutor(max(1, min(8, os.cpu_count() or 1))) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), srcs))
    objs = [o for o, _ in results]
    if verbose:
        for _, log in results:
            if log:
                print(log, file=sys.stderr)
    newest = max(o.stat().st_mtime for o in objs)
    if not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-cudart", "static", "-o",
               str(LIB), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
