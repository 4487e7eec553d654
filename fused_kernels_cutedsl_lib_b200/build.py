"""Build the in-tree shared library ``_lib/libfk_b200.so`` for sm_100a.

Each ``csrc/*.cu`` translation unit is compiled with nvcc
(``-gencode arch=compute_100a,code=sm_100a``) into ``_build/`` and linked into
one C-ABI shared library. The library keeps the CUDA runtime static and
resolves driver entry points (``cuTensorMapEncodeTiled``) at run time, so it
needs no ``-lcuda`` and builds on a machine without a GPU.

Usage: ``python -m fused_kernels_cutedsl_lib_b200.build [--force]``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = REPO_DIR / "_build"
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "libfk_b200.so"
INCLUDE_DIR = REPO_DIR / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    f"-I{INCLUDE_DIR}",
    f"-I{CSRC}",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libfk_b200.so")
    return cand


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))


def _stale(target: Path, inputs: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(p.stat().st_mtime > t for p in inputs)


def _compile_one(nvcc: str, src: Path, verbose: bool) -> Path:
    obj = BUILD_DIR / (src.stem + ".o")
    if not _stale(obj, [src] + _deps()):
        return obj
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        sys.stderr.write(res.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every ``csrc/*.cu`` for sm_100a and link ``libfk_b200.so``."""
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    srcs = _sources()
    if force:
        for o in BUILD_DIR.glob("*.o"):
            o.unlink()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile_one(nvcc, s, verbose), srcs))
    if force or _stale(LIB_PATH, objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-cudart", "static"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


TVMFFI_SRC = PKG_DIR / "tvmffi" / "fk_tvmffi.cc"
TVMFFI_LIB = LIB_DIR / "libfk_b200_tvmffi.so"


def tvm_ffi_paths():
    """(include dirs, lib dir) of the installed apache-tvm-ffi, or None if absent."""
    import importlib.util

    spec = importlib.util.find_spec("tvm_ffi")
    if spec is None or not spec.submodule_search_locations:
        return None
    root = Path(list(spec.submodule_search_locations)[0])
    inc, lib = root / "include", root / "lib"
    if not (inc / "tvm" / "ffi" / "function.h").exists() or not (lib / "libtvm_ffi.so").exists():
        return None
    dl = root / "3rdparty" / "dlpack" / "include"
    incs = [inc] + ([dl] if dl.exists() else [])
    return incs, lib


def build_tvmffi(force: bool = False) -> Path | None:
    """TVM-FFI module over libfk_b200 (skipped when apache-tvm-ffi is not installed)."""
    paths = tvm_ffi_paths()
    if paths is None:
        return None
    incs, libdir = paths
    if not force and not _stale(TVMFFI_LIB, [TVMFFI_SRC, LIB_PATH, INCLUDE_DIR / "fk_b200.h"]):
        return TVMFFI_LIB
    cxx = shutil.which("g++") or "c++"
    cmd = [cxx, "-std=c++17", "-O2", "-fPIC", "-shared", str(TVMFFI_SRC), "-o", str(TVMFFI_LIB),
           f"-I{INCLUDE_DIR}", *[f"-I{i}" for i in incs], f"-L{LIB_DIR}", "-lfk_b200", f"-L{libdir}", "-ltvm_ffi",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{libdir}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"TVM-FFI module build failed:\n{res.stdout}\n{res.stderr}")
    return TVMFFI_LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true", help="print ptxas register usage")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
    print(build_tvmffi(force=args.force))


if __name__ == "__main__":
    main()
