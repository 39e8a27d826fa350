"""Build the native libraries in-tree (``decodekernels_b200/lib/``).

* ``libdk_b200.so``        the CUDA kernels + C ABI (``include/dk_paged_attention.h``),
                           compiled by nvcc for sm_100a only, CUDA runtime linked
                           statically, no torch dependency.
* ``libdk_b200_torch.so``  the ``torch.ops.decode_kernels.paged_attention_decode``
                           registration, compiled by g++ against torch's headers and
                           linked to ``libdk_b200.so`` (rpath ``$ORIGIN``).

Both are rebuilt only when a source is newer than the library.  Run
``python -m decodekernels_b200.build`` or call ``build_all()``.
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
LIB_DIR = PKG / "lib"
INCLUDE = ROOT / "include"

CUDA_LIB = LIB_DIR / "libdk_b200.so"
TORCH_LIB = LIB_DIR / "libdk_b200_torch.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else (shutil.which("nvcc") or "nvcc")


def _cuda_include() -> str:
    return str(Path(_nvcc()).resolve().parent.parent / "include")


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed ({r.returncode}): {cmd[0]} ... {cmd[-1]}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, flush=True)


def cuda_sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "dk_paged_attention.h"]


def build_cuda_library(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """nvcc -> libdk_b200.so (sm_100a, -lineinfo, static cudart)."""
    if not force and not _stale(CUDA_LIB, cuda_sources()):
        return CUDA_LIB
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = CUDA_LIB.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
           "-shared", "-cudart", "static", "-o", str(tmp), str(CSRC / "paged_attention.cu")]
    if ptxas_verbose:
        cmd.insert(1, "-Xptxas=-v")
    _run(cmd, verbose)
    os.replace(tmp, CUDA_LIB)
    return CUDA_LIB


def build_torch_binding(force: bool = False, verbose: bool = False) -> Path:
    """g++ -> libdk_b200_torch.so (registers the decode_kernels torch op)."""
    sources = [CSRC / "torch_binding.cpp", INCLUDE / "dk_paged_attention.h", CUDA_LIB]
    if not force and not _stale(TORCH_LIB, sources):
        return TORCH_LIB
    import torch
    from torch.utils import cpp_extension

    LIB_DIR.mkdir(parents=True, exist_ok=True)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = [f"-I{p}" for p in cpp_extension.include_paths()] + [f"-I{_cuda_include()}"]
    torch_lib = cpp_extension.library_paths()[0]
    tmp = TORCH_LIB.with_suffix(".so.tmp")
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_API_INCLUDE_EXTENSION_H", *incs, str(CSRC / "torch_binding.cpp"), "-o", str(tmp),
           f"-L{LIB_DIR}", "-l:libdk_b200.so", f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch_cpu",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    _run(cmd, verbose)
    os.replace(tmp, TORCH_LIB)
    return TORCH_LIB


def ptxas_report() -> list[dict]:
    """Compile the library's device code once more with ``-Xptxas -v`` (into
    a temporary directory, discarded) and return what ptxas reports for each
    kernel instance: ``name`` (demangled), ``registers``, ``stack_bytes``,
    ``spill_stores``, ``spill_loads``.  The zero-spill check of the test suite
    reads this (DecodeKernels enforces the same per architecture in
    ``tools/compile_check.sh:17-40``)."""
    import re
    import tempfile

    with tempfile.TemporaryDirectory() as tmp:
        cmd = [_nvcc(), *ARCH_FLAGS, "-O3", "-std=c++17", "-cubin", "-Xptxas=-v", "-o",
               str(Path(tmp) / "dk.cubin"), str(CSRC / "paged_attention.cu")]
        r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"ptxas report build failed:\n{r.stdout}{r.stderr}")
    kernels, cur = [], None
    for line in (r.stdout + r.stderr).splitlines():
        m = re.search(r"Compiling entry function '([^']+)'", line)
        if m:
            cur = {"mangled": m.group(1), "registers": None, "stack_bytes": None, "spill_stores": None,
                   "spill_loads": None}
            kernels.append(cur)
            continue
        if cur is None:
            continue
        m = re.search(r"(\d+) bytes stack frame, (\d+) bytes spill stores, (\d+) bytes spill loads", line)
        if m:
            cur["stack_bytes"], cur["spill_stores"], cur["spill_loads"] = (int(x) for x in m.groups())
        m = re.search(r"Used (\d+) registers", line)
        if m:
            cur["registers"] = int(m.group(1))
    names = [k["mangled"] for k in kernels]
    if shutil.which("c++filt") and names:
        out = subprocess.run(["c++filt"], input="\n".join(names), capture_output=True, text=True).stdout.split("\n")
        for k, n in zip(kernels, out):
            k["name"] = n.strip() or k["mangled"]
    for k in kernels:
        k.setdefault("name", k["mangled"])
    return kernels


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_cuda_library(force=force, verbose=verbose)
    build_torch_binding(force=force, verbose=verbose)


if __name__ == "__main__":
    if "--ptxas" in sys.argv:
        for k in ptxas_report():
            print(f"{k['registers']:4d} regs  {k['spill_stores']:3d}/{k['spill_loads']:3d} B spilled  {k['name']}")
    else:
        build_all(force="--force" in sys.argv, verbose=True)
