"""In-tree build of the native parts (sm_100a only).

Two shared objects are produced next to this file:

* ``libnanoserve_sampler.so`` -- the CUDA kernels behind the C ABI declared in
  ``include/nanoserve_sampler.h`` (nvcc, ``-gencode arch=compute_100a,
  code=sm_100a``, static CUDA runtime, no torch dependency);
* ``_nanoserve_ops.so`` -- the torch adapter registering
  ``torch.ops.nanoserve_b200.sample`` (g++ against torch's headers), linked
  to the library above with an ``$ORIGIN`` rpath.

nvcc cross-compiles without a GPU, so ``build()`` works on CPU-only hosts.
"""
from __future__ import annotations

import os
import subprocess
import sysconfig
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
LIB_NAME = "libnanoserve_sampler.so"
OPS_NAME = "_nanoserve_ops.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def _run(cmd: list[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"build step failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile the kernels + C ABI into ``libnanoserve_sampler.so``: every
    ``.cu`` file to an object in parallel (``_build/`` next to this file),
    then one link with the static CUDA runtime."""
    out = PKG_DIR / LIB_NAME
    cus = sorted(CSRC.glob("*.cu"))
    srcs = cus + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE / "nanoserve_sampler.h"]
    if not force and not _stale(out, srcs):
        return out
    objdir = PKG_DIR / "_build"
    objdir.mkdir(exist_ok=True)
    flags = [*ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", f"-I{INCLUDE}"]
    if verbose:
        flags.append("-Xptxas=-v")
    procs = []
    for cu in cus:
        obj = objdir / (cu.stem + ".o")
        cmd = [_nvcc(), *flags, "-c", str(cu), "-o", str(obj)]
        procs.append((cmd, obj, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)))
    objs = []
    for cmd, obj, p in procs:
        so, se = p.communicate()
        if p.returncode != 0:
            raise RuntimeError(f"build step failed: {' '.join(cmd)}\n{so}\n{se}")
        if verbose and se:
            print(se)
        objs.append(str(obj))
    _run([_nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static", *objs, "-o", str(out), "-ldl", "-lrt", "-lpthread"])
    return out


def build_torch_ops(force: bool = False) -> Path:
    """Compile the torch.ops adapter against the installed torch."""
    import torch
    from torch.utils import cpp_extension

    lib = build_library(force=force)
    out = PKG_DIR / OPS_NAME
    src = CSRC / "ns_torch_ops.cpp"
    if not force and not _stale(out, [src, lib, INCLUDE / "nanoserve_sampler.h"]):
        return out
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    incs = cpp_extension.include_paths() + [str(Path(cuda_home) / "include"), str(INCLUDE)]
    torch_lib = str(Path(torch.__file__).resolve().parent / "lib")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [
        "g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        *[f"-I{i}" for i in incs], f"-I{sysconfig.get_paths()['include']}",
        str(src), "-o", str(out),
        f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch_cpu",
        f"-L{PKG_DIR}", "-l:" + LIB_NAME,
        f"-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}",
    ]
    _run(cmd)
    return out


def build(force: bool = False) -> None:
    build_library(force=force)
    build_torch_ops(force=force)


if __name__ == "__main__":
    import sys

    build(force="--force" in sys.argv)
    print("built", PKG_DIR / LIB_NAME, PKG_DIR / OPS_NAME)
