"""Build the in-tree CUDA library ``lib/libecoint8_b200.so`` for sm_100a.

    python eco-int8-opt_b200/build.py [--force] [--verbose]

Compiles every ``csrc/*.cu`` with nvcc (``-gencode arch=compute_100a,code=sm_100a
-lineinfo -O3``) in parallel and links one shared library with the static
CUDA runtime.  The driver API (``cuTensorMapEncodeTiled``) is resolved at run
time through ``cudaGetDriverEntryPoint``, so nothing links against libcuda.
Rebuilds only when a source or header is newer than the library.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIB_DIR = HERE / "lib"
LIB = LIB_DIR / "libecoint8_b200.so"
INCLUDE = HERE.parent / "include"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the ecoint8 B200 library needs the CUDA toolkit to build")


def sources():
    return sorted(CSRC.glob("*.cu"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    newest = max(p.stat().st_mtime for p in [*CSRC.glob("*"), *INCLUDE.glob("*.h")])
    return LIB.stat().st_mtime >= newest


def build(force: bool = False, verbose: bool = False) -> pathlib.Path:
    if not force and up_to_date():
        return LIB
    LIB_DIR.mkdir(exist_ok=True)
    obj_dir = LIB_DIR / "obj"
    obj_dir.mkdir(exist_ok=True)
    cc = nvcc()

    def compile_one(src: pathlib.Path) -> pathlib.Path:
        obj = obj_dir / (src.stem + ".o")
        cmd = [cc, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd += ["-Xptxas", "-v"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stderr}")
        if verbose:
            print(r.stderr, file=sys.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-cudart", "static"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
