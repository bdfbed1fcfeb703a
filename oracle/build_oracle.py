"""Build the CPU checkers (TEST INFRASTRUCTURE ONLY).

    python oracle/build_oracle.py [--ref-root /path/to/OjasX]

The reference tree is taken from --ref-root, else the OJX_REFERENCE_ROOT
environment variable, else a checkout named `reference` beside this repository;
when none of them holds the kernels, oracle/_ref is not built (and the tests that
need it skip).

* oracle/_build/libojx_oracle.so — the C++ restatement (ojx_oracle.cpp), always built.
* oracle/_ref/libref_kernels_nofma.so and libref_kernels_fma.so — the reference's own
  OpenCL C kernels (torchcl/kernels/{matmul,activation,elementwise,precision}.cl, read
  in place from the reference tree) compiled for the host through
  oracle/ref_harness/clshim.h, once with FMA contraction off and once with it on
  (OpenCL leaves `sum += a*b` contraction to the device compiler).  Built only when
  the reference tree is present; nothing from it is copied into this repository.

Flags: -O3 -march=x86-64-v3 (AVX2 + FMA, runs on any recent x86-64 host, unlike
-march=native) -fopenmp.  The restatement is compiled with -ffp-contract=off and
spells the fused variant with explicit fmaf.
"""
from __future__ import annotations

import argparse
import os
import pathlib
import shutil
import subprocess

HERE = pathlib.Path(__file__).resolve().parent
BUILD = HERE / "_build"
REF_OUT = HERE / "_ref"
HARNESS = HERE / "ref_harness"
DEFAULT_REF_ROOT = os.environ.get("OJX_REFERENCE_ROOT") or str(HERE.parent.parent / "reference")
CXX = os.environ.get("OJX_CXX") or ("/usr/bin/g++" if os.path.exists("/usr/bin/g++") else shutil.which("g++") or "g++")
BASE = ["-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared", "-std=c++17"]

ORACLE_LIB = BUILD / "libojx_oracle.so"
REF_LIBS = {"nofma": REF_OUT / "libref_kernels_nofma.so", "fma": REF_OUT / "libref_kernels_fma.so"}


def _run(cmd: list[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")


def _newer(out: pathlib.Path, deps: list[pathlib.Path]) -> bool:
    return out.exists() and all(out.stat().st_mtime >= d.stat().st_mtime for d in deps if d.exists())


def build_oracle(force: bool = False) -> pathlib.Path:
    src = HERE / "ojx_oracle.cpp"
    if not force and _newer(ORACLE_LIB, [src, pathlib.Path(__file__)]):
        return ORACLE_LIB
    BUILD.mkdir(exist_ok=True)
    _run([CXX, *BASE, "-ffp-contract=off", str(src), "-o", str(ORACLE_LIB)])
    return ORACLE_LIB


def ref_kernel_dir(ref_root: str | os.PathLike = DEFAULT_REF_ROOT) -> pathlib.Path:
    return pathlib.Path(ref_root) / "torchcl" / "kernels"


def build_ref(ref_root: str | os.PathLike = DEFAULT_REF_ROOT, force: bool = False) -> dict:
    """Compile the reference kernels; returns {} when the reference tree is absent."""
    kdir = ref_kernel_dir(ref_root)
    cls = {n: kdir / f"{n}.cl" for n in ("matmul", "activation", "elementwise", "precision",
                                          "reduction", "winograd_gemm", "flash_attention")}
    if not all(p.exists() for p in cls.values()):
        return {}
    REF_OUT.mkdir(exist_ok=True)
    srcs = [HARNESS / "ref_kernels.cpp", HARNESS / "fiber.cpp"]
    deps = srcs + [HARNESS / "clshim.h", HARNESS / "fiber.h", pathlib.Path(__file__)] + list(cls.values())
    defs = [f'-DREF_{n.upper()}_CL="{p}"' for n, p in cls.items()]
    for variant, lib in REF_LIBS.items():
        if not force and _newer(lib, deps):
            continue
        contract = "-ffp-contract=off" if variant == "nofma" else "-ffp-contract=fast"
        _run([CXX, *BASE, contract, "-Wno-unknown-pragmas", f"-I{HARNESS}", *defs,
              *map(str, srcs), "-o", str(lib)])
    return dict(REF_LIBS)


def build_ref_jit(cl_file: pathlib.Path, binary: bool, out: pathlib.Path, fma: bool) -> pathlib.Path:
    """Compile one JIT-generated kernel source through the shim (golden generation only)."""
    contract = "-ffp-contract=fast" if fma else "-ffp-contract=off"
    cmd = [CXX, *BASE, contract, "-Wno-unknown-pragmas", f"-I{HARNESS}", f'-DREF_JIT_CL="{cl_file}"']
    if binary:
        cmd.append("-DREF_JIT_BINARY")
    _run(cmd + [str(HARNESS / "ref_jit.cpp"), str(HARNESS / "fiber.cpp"), "-o", str(out)])
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-root", default=DEFAULT_REF_ROOT)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build_oracle(a.force))
    refs = build_ref(a.ref_root, a.force)
    print(refs if refs else "reference tree not found: oracle/_ref not built")
