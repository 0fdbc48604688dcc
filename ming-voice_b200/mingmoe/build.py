"""Build the C-ABI library `libmingmoe.so` from `csrc/*.cu` with nvcc, in-tree, for sm_100a only.

    python ming-voice_b200/mingmoe/build.py [-v] [--force]

Each translation unit compiles to an object under `mingmoe/_build/` (skipped when up to date), then they
link into `mingmoe/libmingmoe.so` next to this file. The CUDA runtime is linked statically, so the library
depends only on the driver.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
CSRC = os.path.join(PKG, "csrc")
ROOT = os.path.dirname(PKG)
INCLUDE = os.path.join(ROOT, "include")
OUT = os.path.join(HERE, "libmingmoe.so")
BUILD = os.path.join(HERE, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xcompiler", "-fvisibility=hidden", "-I", CSRC, "-I", INCLUDE]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _deps():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) +
                  glob.glob(os.path.join(INCLUDE, "*.h")))


def _compile(src: str, verbose: bool, ptxas_v: bool, build_dir: str = BUILD, extra=()) -> str:
    obj = os.path.join(build_dir, os.path.basename(src) + ".o")
    newest_dep = max([os.path.getmtime(src)] + [os.path.getmtime(d) for d in _deps()])
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest_dep and not ptxas_v:
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
    if ptxas_v:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if ptxas_v or verbose:
        sys.stdout.write(r.stderr)
    return obj


def build(verbose: bool = False, force: bool = False, ptxas_v: bool = False, out: str = OUT, build_dir: str = BUILD,
          extra=()) -> str:
    """Compile and link; `out`, `build_dir` and `extra` nvcc flags select a variant build (e.g. -DMV_TRACE for
    the phase-timing stamps of the decode kernel) without touching the default library."""
    OUT = out
    os.makedirs(build_dir, exist_ok=True)
    if force:
        for f in glob.glob(os.path.join(build_dir, "*.o")):
            os.remove(f)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, ptxas_v, build_dir, tuple(extra)), srcs))
    if (not os.path.exists(OUT) or force or ptxas_v or
            max(os.path.getmtime(o) for o in objs) > os.path.getmtime(OUT)):
        tmp = OUT + ".tmp"
        cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-cudart", "static"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="--force" in sys.argv, ptxas_v="--ptxas" in sys.argv))
