"""Build libojx.so (the sm_100a kernels + C-ABI runtime) in-tree, and its
bounds-checking twin libojx_debug.so (-DOJX_DEBUG_BOUNDS).

    python ojasx-open-source-cuda-_b200/build.py [--verbose-ptxas]

Compiles csrc/ojx_kernels.cu (every kernel, one translation unit), csrc/runtime.cpp,
csrc/tmap.cpp and csrc/graph.cpp with nvcc for `-gencode arch=compute_100a,code=sm_100a` and links
them into ojasx-open-source-cuda-_b200/torchcl/_lib/libojx.so, next to the Python
package that loads it.  The CUDA runtime is linked statically, so the library does
not depend on which libcudart another module (e.g. torch) already loaded.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
OUT_DIR = PKG / "torchcl" / "_lib"
OBJ_DIR = PKG / "_build"
LIB = OUT_DIR / "libojx.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", f"-I{INCLUDE}", f"-I{CSRC}"]
SOURCES = ["ojx_kernels.cu", "runtime.cpp", "tmap.cpp", "graph.cpp"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


# Two builds of the same sources: the library itself, and the bounds-checking build
# (every TMA tile origin and epilogue store checked on the device; torchcl loads it
# when OJX_DEBUG_BOUNDS=1).
VARIANTS = {"release": (LIB, OBJ_DIR, []),
            "debug": (OUT_DIR / "libojx_debug.so", OBJ_DIR / "debug", ["-DOJX_DEBUG_BOUNDS"])}


def _compile(src: str, obj_dir: pathlib.Path, defs: list[str], verbose_ptxas: bool) -> pathlib.Path:
    obj = obj_dir / (pathlib.Path(src).stem + ".o")
    cmd = [nvcc(), *ARCH, *COMMON, *defs, "-c", str(CSRC / src), "-o", str(obj)]
    if verbose_ptxas and src.endswith(".cu"):
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    if verbose_ptxas and res.stderr:
        (obj_dir / (pathlib.Path(src).stem + ".ptxas.txt")).write_text(res.stderr)
    return obj


def _stale(lib: pathlib.Path) -> bool:
    if not lib.exists():
        return True
    t = lib.stat().st_mtime
    deps = list(CSRC.glob("*")) + list(INCLUDE.glob("*.h")) + [pathlib.Path(__file__)]
    return any(p.stat().st_mtime > t for p in deps)


def _link(lib: pathlib.Path, objs: list[pathlib.Path]) -> None:
    tmp = lib.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-ldl"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, lib)


def build(force: bool = False, verbose_ptxas: bool = False) -> pathlib.Path:
    """Build every stale variant (both compile in parallel); returns the release library."""
    todo = {name: v for name, v in VARIANTS.items() if force or _stale(v[0])}
    if not todo:
        return LIB
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    jobs = []
    for name, (lib, obj_dir, defs) in todo.items():
        obj_dir.mkdir(parents=True, exist_ok=True)
        jobs += [(name, src, obj_dir, defs) for src in SOURCES]
    with cf.ThreadPoolExecutor(max_workers=len(jobs)) as ex:
        objs = list(ex.map(lambda j: (j[0], _compile(j[1], j[2], j[3], verbose_ptxas)), jobs))
    for name, (lib, _, _) in todo.items():
        _link(lib, [o for n, o in objs if n == name])
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force or a.verbose_ptxas, verbose_ptxas=a.verbose_ptxas))
    sys.exit(0)
