"""Build ``libatomb200.so`` (the C-ABI kernel library) in-tree with nvcc for sm_100a.

    python -m tt_atom.build            # or build() from Python

The library is written next to this file so it travels with the source tree; ``_lib.py`` loads
it from there and refuses to run without it.
"""
from __future__ import annotations

import os
import pathlib
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = pathlib.Path(__file__).resolve().parent
CSRC = PKG.parent / "csrc"
INCLUDE = PKG.parent.parent / "include"
LIB = PKG / "libatomb200.so"
OBJ = PKG.parent / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         f"-I{INCLUDE}"]


def _nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and pathlib.Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(CSRC.glob("*.cu"))


def _stale(obj, src):
    if not obj.exists():
        return True
    deps = [src, *CSRC.glob("*.cuh"), *INCLUDE.glob("*.h")]
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def build(verbose=False, ptxas_info=False):
    nvcc = _nvcc()
    OBJ.mkdir(exist_ok=True)
    srcs = sources()
    objs = [OBJ / (s.stem + ".o") for s in srcs]

    def compile_one(so):
        s, o = so
        if not _stale(o, s) and not ptxas_info:
            return None
        cmd = [nvcc, *ARCH, *FLAGS, "-c", str(s), "-o", str(o)]
        if ptxas_info:
            cmd += ["-Xptxas", "-v"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {s.name}:\n{r.stderr}")
        return r.stderr if (verbose or ptxas_info) else None

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for out in ex.map(compile_one, zip(srcs, objs)):
            if out:
                print(out, file=sys.stderr)
    if not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [nvcc, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_info="-v" in sys.argv)
    print(LIB)
