"""Build recipe for the package's native code (in-tree, sm_100a only).

Two shared objects are produced next to this file:

* ``libfp8linear_b200.so`` -- the CUDA kernels and the C ABI of
  ``include/fp8linear_b200.h``; built by nvcc with
  ``-gencode arch=compute_100a,code=sm_100a`` and the shared CUDA runtime (so the
  current device/stream state is the one torch uses).
* ``_C.so`` -- the thin torch binding (TORCH_LIBRARY ``fp8linear_b200``) that
  calls the C ABI; loaded with ``torch.ops.load_library``.

``python fp8linear_b200/_build.py`` (or ``build()``) rebuilds what is stale; it is a
plain script so it runs before the package (whose import needs the binding) can load.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB = PKG / "libfp8linear_b200.so"
BINDING = PKG / "_C.so"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

KERNEL_SOURCES = ["quantize.cu", "gemm_sm100.cu", "gemm_small_sm100.cu", "capi.cu", "noalloc.cu"]
HEADERS = ["ptx.cuh", "internal.h"]


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed ({r.returncode}): {' '.join(cmd[:3])} ...")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr)


def _torch_paths():
    import torch
    from torch.utils import cpp_extension

    inc = cpp_extension.include_paths()
    libdir = str(Path(torch.__file__).resolve().parent / "lib")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    return inc, libdir, abi


def build_kernels(verbose: bool = False, ptxas_info: bool = False) -> Path:
    deps = [CSRC / s for s in KERNEL_SOURCES + HEADERS] + [INCLUDE / "fp8linear_b200.h",
                                                           Path(__file__)]
    if not _stale(LIB, deps):
        return LIB
    tmp = LIB.with_name(LIB.name + f".tmp{os.getpid()}")
    cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
           "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-shared",
           "-cudart", "shared", f"-I{INCLUDE}",
           *[str(CSRC / s) for s in KERNEL_SOURCES],
           "-o", str(tmp),
           f"-Xlinker", f"-rpath,{CUDA_HOME / 'lib64'}", "-Xlinker", "-soname,libfp8linear_b200.so"]
    if ptxas_info:
        cmd.insert(1, "-Xptxas=-v")
    _run(cmd, verbose)
    os.replace(tmp, LIB)
    return LIB


def build_binding(verbose: bool = False) -> Path:
    deps = [CSRC / "torch_binding.cpp", INCLUDE / "fp8linear_b200.h", LIB, Path(__file__)]
    if not _stale(BINDING, deps):
        return BINDING
    inc, libdir, abi = _torch_paths()
    # The system g++ links libstdc++ dynamically. A compiler that embeds a static
    # libstdc++ in the binding breaks C++ exceptions thrown by torch (TORCH_CHECK)
    # when they unwind through the binding's frames.
    cxx = os.environ.get("FP8LIN_CXX") or ("/usr/bin/g++" if Path("/usr/bin/g++").exists()
                                           else shutil.which("g++") or "g++")
    tmp = BINDING.with_name(BINDING.name + f".tmp{os.getpid()}")
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *[f"-isystem{p}" for p in inc], f"-isystem{CUDA_HOME / 'include'}",
           f"-I{INCLUDE}", str(CSRC / "torch_binding.cpp"), "-o", str(tmp),
           f"-L{libdir}", f"-L{PKG}", "-lfp8linear_b200", "-lc10", "-lc10_cuda", "-ltorch",
           "-ltorch_cpu", "-ltorch_cuda",
           f"-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{libdir}", f"-Wl,-rpath,{CUDA_HOME / 'lib64'}"]
    _run(cmd, verbose)
    needed = subprocess.run(["readelf", "-d", str(tmp)], capture_output=True, text=True).stdout
    if "libstdc++" not in needed:
        os.unlink(tmp)
        raise RuntimeError(f"{cxx} linked libstdc++ statically into the torch binding; "
                           "set FP8LIN_CXX to a g++ that links it dynamically")
    os.replace(tmp, BINDING)
    return BINDING


def build(verbose: bool = False) -> None:
    build_kernels(verbose)
    build_binding(verbose)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(LIB)
    print(BINDING)
