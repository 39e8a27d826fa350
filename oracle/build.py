"""Build recipe for the checkers under oracle/ (test infrastructure).

* ``build_oracle()``            gcc -O2 -fopenmp paged_attention_cpu.c
                                -> oracle/_build/libdk_oracle.so
* ``build_reference_kernel()``  nvcc sm_100a ref_kernel_shim.cu with the
                                DecodeKernels tree's ``csrc/`` on the include
                                path -> oracle/_ref/libdk_ref_kernel.so.  Runs
                                only where that tree exists (``DK_REFERENCE_DIR``,
                                else a ``reference`` directory beside this
                                repository's checkout); elsewhere
                                it keeps a prebuilt library if one is present.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
BUILD = HERE / "_build"
REF_OUT = HERE / "_ref"
ORACLE_LIB = BUILD / "libdk_oracle.so"
REF_LIB = REF_OUT / "libdk_ref_kernel.so"


def _stale(target: Path, sources: list[Path]) -> bool:
    return not target.exists() or any(s.stat().st_mtime > target.stat().st_mtime for s in sources)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"oracle build failed: {' '.join(cmd)}")


def build_oracle(force: bool = False) -> Path:
    src = HERE / "paged_attention_cpu.c"
    if force or _stale(ORACLE_LIB, [src]):
        BUILD.mkdir(exist_ok=True)
        tmp = ORACLE_LIB.with_suffix(".so.tmp")
        _run(["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-std=c11", str(src), "-o", str(tmp), "-lm"])
        os.replace(tmp, ORACLE_LIB)
    return ORACLE_LIB


def reference_dir() -> Path:
    """The DecodeKernels source tree: ``DK_REFERENCE_DIR``, else ``../reference``
    relative to this repository's root."""
    env = os.environ.get("DK_REFERENCE_DIR")
    return Path(env) if env else HERE.parent.parent / "reference"


def build_reference_kernel(force: bool = False) -> Path | None:
    ref_csrc = reference_dir() / "csrc"
    header = ref_csrc / "paged_attention.cuh"
    shim = HERE / "ref_kernel_shim.cu"
    if not header.exists():
        return REF_LIB if REF_LIB.exists() else None
    if force or _stale(REF_LIB, [shim, header, ref_csrc / "common.cuh"]):
        REF_OUT.mkdir(exist_ok=True)
        nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
        nvcc = nvcc if os.path.exists(nvcc) else (shutil.which("nvcc") or "nvcc")
        tmp = REF_LIB.with_suffix(".so.tmp")
        _run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17", "-I",
              str(ref_csrc), "-Xcompiler", "-fPIC", "-shared", "-cudart", "static", str(shim), "-o", str(tmp)])
        os.replace(tmp, REF_LIB)
    return REF_LIB


if __name__ == "__main__":
    print(build_oracle(force=True))
    print(build_reference_kernel(force=True))
