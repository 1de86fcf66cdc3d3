"""TEST INFRASTRUCTURE ONLY.  Build recipe for the parity checkers.

* ``oracle/_build/liboracle.so``  the plain-C restatement (gdsq_oracle.c),
  gcc -O2 with OpenMP.  Built everywhere.
* ``oracle/_ref/libref_kernels.so``  GdsLLM's own CUDA kernels compiled
  unchanged from the reference tree (gdsllm/runtime/fused_gemv.cu,
  gguf_dequant.cu, affine_q4_dequant.cu) for sm_100a, plus ref_shim.cu.
  Built only where the reference tree is present; the product travels to the
  GPU box without it.  Nothing from the reference tree is copied into this
  repository: nvcc reads the sources where they lie.

Run ``python oracle/build.py [--force]``.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

ORACLE = Path(__file__).resolve().parent
BUILD = ORACLE / "_build"
REF_OUT = ORACLE / "_ref"
ORACLE_LIB = BUILD / "liboracle.so"
REF_LIB = REF_OUT / "libref_kernels.so"
# The reference checkout: $GDSLLM_REFERENCE, else a directory named
# "reference" next to this repository.
REFERENCE_ROOT = Path(os.environ.get("GDSLLM_REFERENCE", ORACLE.parent.parent / "reference"))
REFERENCE_RUNTIME = REFERENCE_ROOT / "gdsllm" / "runtime"
REF_SOURCES = ["fused_gemv.cu", "gguf_dequant.cu", "affine_q4_dequant.cu"]
NVCC = str(Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc")


def _stale(target: Path, sources) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(s).stat().st_mtime > t for s in sources)


def build_oracle(force: bool = False) -> Path:
    src = ORACLE / "gdsq_oracle.c"
    if force or _stale(ORACLE_LIB, [src]):
        BUILD.mkdir(exist_ok=True)
        tmp = ORACLE_LIB.with_suffix(".tmp")
        # -ffp-contract=off: the only fused multiply-add is the explicit fmaf.
        subprocess.run(["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
                        "-o", str(tmp), str(src), "-lm"], check=True)
        os.replace(tmp, ORACLE_LIB)
    return ORACLE_LIB


def build_reference_kernels(force: bool = False) -> Path | None:
    """Compiles the reference kernels; returns None when the tree is absent."""
    if not REFERENCE_RUNTIME.is_dir():
        return REF_LIB if REF_LIB.exists() else None
    sources = [REFERENCE_RUNTIME / s for s in REF_SOURCES] + [ORACLE / "ref_shim.cu"]
    if force or _stale(REF_LIB, sources):
        REF_OUT.mkdir(exist_ok=True)
        tmp = REF_LIB.with_suffix(".tmp")
        # The reference's setup.py passes only -std=c++17 (setup.py:120-123), so
        # nvcc's defaults (including FMA contraction) apply, as they do here.
        subprocess.run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                        "-Xcompiler", "-fPIC", "-shared", "-I", str(REFERENCE_RUNTIME),
                        "-o", str(tmp), *[str(s) for s in sources]], check=True)
        os.replace(tmp, REF_LIB)
    return REF_LIB


REF_PACKAGE = ORACLE.parent / "baseline" / "_ref"


def install_reference_package(force: bool = False) -> Path | None:
    """Installs the reference package (its Python modules and its compiled
    extension) into baseline/_ref, the one offline pip install this project
    makes, so that tests can run the reference's own callers (llama.py,
    scheduler.py, qwen_moe.py).  The build writes into its source tree, so it
    runs on a copy under the system temporary directory.  Returns the target,
    or None when the reference tree is absent."""
    import shutil
    import tempfile

    if (REF_PACKAGE / "gdsllm" / "runtime" / "scheduler.py").exists() and not force:
        return REF_PACKAGE
    if not REFERENCE_RUNTIME.is_dir():
        return None
    with tempfile.TemporaryDirectory() as tmp:
        src = Path(tmp) / "reference"
        shutil.copytree(REFERENCE_ROOT, src)
        env = dict(os.environ, TORCH_CUDA_ARCH_LIST="10.0a")
        subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
                        "--find-links", "/opt/wheelhouse", "--upgrade", "--target", str(REF_PACKAGE), str(src)],
                       check=True, env=env)
    return REF_PACKAGE


if __name__ == "__main__":
    force = "--force" in sys.argv
    print(build_oracle(force))
    print(build_reference_kernels(force))
    print(install_reference_package(force))
