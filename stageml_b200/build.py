"""Build the native libraries of stageml_b200 in-tree (no JIT cache).

  lib/libstageml_b200.so     CUDA kernels + the C ABI of include/stageml_b200.h
                             (nvcc, -gencode arch=compute_100a,code=sm_100a)
  lib/libstageml_torch.so    the `stageml` torch custom-op library, a thin C++
                             layer over the C ABI (g++ against torch's headers)

Run ``python -m stageml_b200.build`` or call :func:`build`. Objects are rebuilt
only when a source or header is newer than the library.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIBDIR = PKG / "lib"
INCLUDE = PKG.parent / "include"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))

CU_SOURCES = [
    "host_util.cu",
    "route.cu",
    "permute.cu",
    "shrink.cu",
    "shrink_tc.cu",
    "grouped_gemm.cu",
    "grouped_gemm_pair.cu",
    "skinny.cu",
    "ep.cu",
    "combine.cu",
    "fold.cu",
    "gemv.cu",
    "fp8.cu",
    "stage_timer.cu",
    "capi.cu",
]
NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
]

CORE_LIB = LIBDIR / "libstageml_b200.so"
TORCH_LIB = LIBDIR / "libstageml_torch.so"


def _newest(paths) -> float:
    return max(p.stat().st_mtime for p in paths)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    res = subprocess.run([str(c) for c in cmd], capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} (exit {res.returncode})")


def build_core(force: bool = False, verbose: bool = False) -> Path:
    """Compile the CUDA sources into lib/libstageml_b200.so."""
    LIBDIR.mkdir(exist_ok=True)
    objdir = LIBDIR / "obj"
    objdir.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [INCLUDE / "stageml_b200.h"]
    hdr_time = _newest(headers)
    nvcc = str(CUDA_HOME / "bin" / "nvcc")
    objs = []
    procs = []
    for src in CU_SOURCES:
        s = CSRC / src
        o = objdir / (src + ".o")
        objs.append(o)
        if force or not o.exists() or o.stat().st_mtime < max(s.stat().st_mtime, hdr_time):
            cmd = [nvcc, *NVCC_FLAGS, "-c", str(s), "-o", str(o)]
            if verbose:
                print(" ".join(cmd), flush=True)
            procs.append((cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = []
    for cmd, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            failed.append((cmd, out))
    if failed:
        for cmd, out in failed:
            sys.stderr.write(" ".join(cmd) + "\n" + out)
        raise RuntimeError("nvcc failed")
    if force or not CORE_LIB.exists() or CORE_LIB.stat().st_mtime < _newest(objs):
        # symbols stay hidden except the extern "C" API, which is exported explicitly
        _run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(CORE_LIB), *map(str, objs),
              "-Xlinker", f"--version-script={CSRC / 'exports.map'}"], verbose)
    return CORE_LIB


def build_torch_ops(force: bool = False, verbose: bool = False) -> Path:
    """Compile csrc/torch_ops.cpp into lib/libstageml_torch.so (links libstageml_b200.so)."""
    import torch
    from torch.utils import cpp_extension

    src = CSRC / "torch_ops.cpp"
    deps = [src, INCLUDE / "stageml_b200.h", CORE_LIB]
    if not force and TORCH_LIB.exists() and TORCH_LIB.stat().st_mtime >= _newest(deps):
        return TORCH_LIB
    incs = cpp_extension.include_paths() + [str(CUDA_HOME / "include")]
    libdirs = cpp_extension.library_paths()
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=stageml_torch", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    cmd += [f"-I{p}" for p in incs]
    cmd += [str(src), "-o", str(TORCH_LIB)]
    cmd += [f"-L{p}" for p in libdirs] + [f"-Wl,-rpath,{p}" for p in libdirs]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda"]
    cmd += [f"-L{LIBDIR}", "-lstageml_b200", "-Wl,-rpath,$ORIGIN"]
    _run(cmd, verbose)
    return TORCH_LIB


def build(force: bool = False, verbose: bool = False) -> None:
    build_core(force=force, verbose=verbose)
    build_torch_ops(force=force, verbose=verbose)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
