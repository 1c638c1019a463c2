"""Ahead-of-time build of the warp_decode_b200 native code, in-tree.

Two artefacts are produced next to this file:

* ``libwarp_decode_b200.so`` -- the C ABI (``include/warp_decode.h``) and all
  CUDA kernels, compiled by nvcc for sm_100a only, with the CUDA runtime
  linked statically.  No PyTorch dependency.
* ``_wd_ext<EXT_SUFFIX>`` -- the PyTorch extension (``csrc/binding.cpp``) that
  exposes the reference's ``moe_gate_up_3d_batched`` / ``moe_down_3d_batched``
  API on top of the C ABI; linked against the library above via an
  ``$ORIGIN`` rpath.

The reference JIT-compiles on import (``__init__.py:36-43`` of
Religious-J/warp_decode).  Here the build is explicit and the import never
compiles, so a machine without nvcc can use a prebuilt tree.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB_NAME = "warp_decode_b200"
LIB = PKG / f"lib{LIB_NAME}.so"
EXT_NAME = "_wd_ext"
EXT = PKG / (EXT_NAME + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "-shared",
    "-cudart", "static",
    "--expt-relaxed-constexpr",
]

LIB_SOURCES = [CSRC / "wd_lib.cu"]
LIB_DEPS = LIB_SOURCES + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "warp_decode.h"]
EXT_SOURCES = [CSRC / "binding.cpp"]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _run(cmd, verbose: bool) -> None:
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    res = subprocess.run([str(c) for c in cmd], capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(
            f"build command failed ({res.returncode}):\n{' '.join(map(str, cmd))}\n"
            f"{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)


def build_lib(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile the C-ABI library (all CUDA kernels) for sm_100a."""
    if force or _stale(LIB, LIB_DEPS):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [_nvcc()] + NVCC_FLAGS + ["-I", INCLUDE, "-o", tmp] + LIB_SOURCES
        if ptxas_verbose:
            cmd.insert(1, "-Xptxas=-v")
        _run(cmd, verbose or ptxas_verbose)
        os.replace(tmp, LIB)
    return LIB


def build_ext(force: bool = False, verbose: bool = False) -> Path:
    """Compile the PyTorch extension against the C-ABI library."""
    import torch
    from torch.utils import cpp_extension

    deps = EXT_SOURCES + [INCLUDE / "warp_decode.h", LIB]
    if force or _stale(EXT, deps):
        cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
        abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
        inc = [INCLUDE, Path(cuda_home) / "include", sysconfig.get_paths()["include"]]
        inc += [Path(p) for p in cpp_extension.include_paths()]
        libdirs = [Path(p) for p in cpp_extension.library_paths()]
        tmp = EXT.with_suffix(".tmp")
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared",
               f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
               f"-DTORCH_EXTENSION_NAME={EXT_NAME}", "-DTORCH_API_INCLUDE_EXTENSION_H"]
        cmd += [f"-I{p}" for p in inc]
        cmd += [str(s) for s in EXT_SOURCES]
        cmd += ["-o", str(tmp), f"-L{PKG}", f"-l{LIB_NAME}", "-Wl,-rpath,$ORIGIN"]
        for d in libdirs:
            cmd += [f"-L{d}", f"-Wl,-rpath,{d}"]
        cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python"]
        _run(cmd, verbose)
        os.replace(tmp, EXT)
    return EXT


def build(force: bool = False, verbose: bool = False) -> None:
    build_lib(force=force, verbose=verbose)
    build_ext(force=force, verbose=verbose)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
