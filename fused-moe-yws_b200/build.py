"""In-tree build of the fused MoE library for sm_100a.

Produces, inside ``fused-moe-yws_b200/lib``:

* ``libfmoe.so`` -- the CUDA kernels plus the C ABI of ``include/fmoe.h``
  (nvcc, ``-gencode arch=compute_100a,code=sm_100a``, no fast-math: the routing kernel
  relies on IEEE single-precision rounding).
* ``libfmoe_tvm_ffi.so`` -- the TVM-FFI ``kernel`` export with the reference signature,
  built only when the ``tvm_ffi`` headers are importable.

Run ``python fused-moe-yws_b200/build.py`` or call ``build()``.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "lib"
INCLUDE = PKG.parent / "include"
OBJ = PKG / "_build"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              f"-I{INCLUDE}", "-Xptxas", "-v"]
CU_SOURCES = ["route.cu", "permute.cu", "gemm_sm100.cu", "gemm_sm100_tm.cu", "fmoe_api.cu", "ep.cu",
              "route_static.cu", "selftest.cu"]


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _headers():
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [INCLUDE / "fmoe.h"]


def _compile(src: str, verbose: bool) -> Path:
    obj = OBJ / (Path(src).stem + ".o")
    deps = [CSRC / src] + _headers()
    if _stale(obj, deps):
        cmd = [NVCC, *ARCH, *NVCC_FLAGS, "-c", str(CSRC / src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        (OBJ / (Path(src).stem + ".ptxas.txt")).write_text(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr[-4000:]}")
        if verbose:
            print(f"[fmoe build] compiled {src}")
    return obj


def build_core(verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    LIB.mkdir(exist_ok=True)
    with ThreadPoolExecutor(max_workers=len(CU_SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), CU_SOURCES))
    so = LIB / "libfmoe.so"
    if _stale(so, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(so), *map(str, objs), "-lcudart"]
        subprocess.check_call(cmd)
        if verbose:
            print(f"[fmoe build] linked {so}")
    return so


def build_tvm_ffi(verbose: bool = False):
    try:
        import tvm_ffi  # noqa: F401
        from tvm_ffi import libinfo
    except Exception:  # pragma: no cover - optional binding
        return None
    inc = [f"-I{p}" for p in libinfo.include_paths()]
    libdir = Path(libinfo.find_libtvm_ffi()).parent
    src = CSRC / "tvm_ffi_kernel.cc"
    so = LIB / "libfmoe_tvm_ffi.so"
    if _stale(so, [src, INCLUDE / "fmoe.h", LIB / "libfmoe.so"]):
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", str(src), "-o", str(so),
               f"-I{INCLUDE}", f"-I{CUDA_HOME / 'include'}", *inc, f"-L{LIB}", "-lfmoe",
               f"-L{libdir}", "-ltvm_ffi", f"-L{CUDA_HOME / 'lib64'}", "-lcudart",
               "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{libdir}"]
        subprocess.check_call(cmd)
        if verbose:
            print(f"[fmoe build] linked {so}")
    return so


def build(verbose: bool = False):
    so = build_core(verbose)
    tvm = build_tvm_ffi(verbose)
    return so, tvm


if __name__ == "__main__":
    print(build(verbose=True))
    sys.exit(0)
