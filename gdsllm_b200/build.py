"""Builds the native parts of gdsllm_b200 in-tree.

* ``_build/libgdsq.so``        every CUDA kernel plus the C ABI of include/gdsq.h,
                               compiled by nvcc for sm_100a only.
* ``_build/gds_io_ext*.so``    the torch binding that mirrors the reference's
                               ``gdsllm.runtime.gds_io_ext`` module, linked
                               against libgdsq.so.

Both are rebuilt only when a source is newer than the product.  Run
``python -m gdsllm_b200.build`` (``--force`` to rebuild everything).
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
INCLUDE = PKG.parent / "include"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-Xlinker", "--exclude-libs,ALL",
    "-Xlinker", "-soname=libgdsq.so",
]

LIB_PATH = BUILD / "libgdsq.so"
EXT_PATH = BUILD / ("gds_io_ext" + sysconfig.get_config_var("EXT_SUFFIX"))


def _newer(target: Path, sources) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(s).stat().st_mtime > t for s in sources)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True)


def build_lib(force: bool = False, verbose: bool = True) -> Path:
    sources = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    if force or _newer(LIB_PATH, sources):
        BUILD.mkdir(parents=True, exist_ok=True)
        tmp = LIB_PATH.with_suffix(".so.tmp")
        _run([NVCC, *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-shared", "-o", tmp,
              CSRC / "gdsq.cu"], verbose)
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def build_ext(force: bool = False, verbose: bool = True) -> Path:
    import torch
    from torch.utils import cpp_extension

    sources = [CSRC / "gds_io_ext.cpp", INCLUDE / "gdsq.h", LIB_PATH]
    if not (force or _newer(EXT_PATH, sources)):
        return EXT_PATH
    BUILD.mkdir(parents=True, exist_ok=True)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    includes = []
    for p in cpp_extension.include_paths():
        includes += ["-I", p]
    includes += ["-I", str(CUDA_HOME / "include"), "-I", sysconfig.get_paths()["include"],
                 "-I", str(INCLUDE)]
    torch_lib = str(Path(torch.__file__).parent / "lib")
    tmp = EXT_PATH.with_suffix(".tmp")
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden",
           "-DTORCH_EXTENSION_NAME=gds_io_ext", "-DTORCH_API_INCLUDE_EXTENSION_H",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", *includes,
           str(CSRC / "gds_io_ext.cpp"), "-o", str(tmp),
           f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
           "-ltorch_python", f"-L{BUILD}", "-lgdsq", "-Wl,-rpath,$ORIGIN",
           f"-L{CUDA_HOME / 'lib64'}", "-lcudart", "-ldl"]
    _run(cmd, verbose)
    os.replace(tmp, EXT_PATH)
    return EXT_PATH


def build_all(force: bool = False, verbose: bool = True) -> None:
    build_lib(force, verbose)
    build_ext(force, verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
