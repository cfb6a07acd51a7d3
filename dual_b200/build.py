"""In-tree build of the C-ABI library ``dual_b200/lib/libdual_b200.so`` (sm_100a).

The library is compiled with nvcc directly (no torch extension machinery), so the
same .so is what the Python wrappers load through ctypes and what a C/C++
caller links against via ``include/dual_b200.h``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIBDIR = PKG / "lib"
LIBNAME = "libdual_b200.so"
SUPPLIER = "dual_supplier"  # native KV-supplier process (supplier_service.cpp)
SOURCES = ["capi.cu", "decode.cu", "decode_noalloc.cu", "pack.cu", "migrate.cu", "prefill.cu", "stage.cu", "kv_write.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the dual_b200 CUDA library cannot be built")


def library_path() -> Path:
    return LIBDIR / LIBNAME


def _stale(target: Path) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    deps = (list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(CSRC.glob("*.cpp"))
            + [ROOT / "include" / "dual_b200.h"])
    return any(d.stat().st_mtime > mtime for d in deps if d.exists())


def supplier_path() -> Path:
    return LIBDIR / SUPPLIER


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile every CUDA source into the shared library and the native supplier executable
    (skipped when up to date)."""
    target = library_path()
    if not force and not _stale(target) and not _stale(supplier_path()):
        return target
    LIBDIR.mkdir(parents=True, exist_ok=True)
    objdir = ROOT / "_build" / "obj"
    objdir.mkdir(parents=True, exist_ok=True)
    common = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              "--expt-relaxed-constexpr", "-I", str(ROOT / "include")]
    if ptxas_verbose:
        common += ["-Xptxas", "-v"]
    objs = []
    for src in SOURCES:
        obj = objdir / (Path(src).stem + ".o")
        cmd = [*common, "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
        if ptxas_verbose or verbose:
            sys.stderr.write(res.stderr)
        objs.append(str(obj))
    tmp = target.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *objs, "-cudart", "static"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    tmp.replace(target)
    exe_tmp = LIBDIR / (SUPPLIER + ".tmp")
    cmd = [nvcc(), *ARCH, "-O2", "-std=c++17", "-I", str(ROOT / "include"), str(CSRC / "supplier_service.cpp"),
           "-o", str(exe_tmp), "-cudart", "static"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"dual_supplier build failed:\n{res.stdout}\n{res.stderr}")
    exe_tmp.replace(supplier_path())
    return target


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_verbose="-v" in sys.argv)
    print(library_path())
