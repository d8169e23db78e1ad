"""Build the sm_100a shared library `libduplex_b200.so` in-tree with nvcc.

    python -m duplex._build            (from qwen3-omni-duplex_b200/)

The library depends only on the CUDA runtime (linked statically by nvcc); it has
no PyTorch symbols, so the C ABI in include/duplex_b200.h can be bound from any
host language.  Rebuilds only when a source is newer than the library.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent                      # qwen3-omni-duplex_b200/
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"
LIB = PKG / "libduplex_b200.so"
TORCH_OPS_SRC = CSRC / "torch_ops.cpp"
TORCH_OPS_LIB = PKG / "libduplex_torch_ops.so"
ARCH = "-gencode=arch=compute_100a,code=sm_100a"


def sources():
    return sorted(CSRC.glob("*.cu"))


def deps():
    return sources() + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def nvcc_path():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libduplex_b200.so")


def needs_build(lib: Path = LIB) -> bool:
    if not lib.exists():
        return True
    t = lib.stat().st_mtime
    return any(p.stat().st_mtime > t for p in deps())


def _compile(src: Path, obj: Path, verbose: bool) -> str:
    cmd = [nvcc_path(), ARCH, "-O3", "-lineinfo", "-std=c++17", "-c",
           "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
           f"-I{INCLUDE}", f"-I{CSRC}", "-o", str(obj), str(src)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


def build(force: bool = False, verbose: bool = False, lib: Path = LIB) -> Path:
    """Compile every csrc/*.cu for sm_100a (one nvcc process per file, in parallel)
    and link them into the shared library."""
    if not force and not needs_build(lib):
        return lib
    from concurrent.futures import ThreadPoolExecutor
    import tempfile
    with tempfile.TemporaryDirectory(prefix="duplex_build_") as tmpd:
        objs = [Path(tmpd) / (s.stem + ".o") for s in sources()]
        with ThreadPoolExecutor(max(1, min(len(objs), os.cpu_count() or 1))) as ex:
            logs = list(ex.map(lambda so: _compile(so[0], so[1], verbose), zip(sources(), objs)))
        tmp = lib.with_suffix(".so.tmp")
        cmd = [nvcc_path(), ARCH, "--shared", "-o", str(tmp)] + [str(o) for o in objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("nvcc link failed:\n" + r.stdout + r.stderr)
    if verbose:
        sys.stderr.write("".join(logs))
    os.replace(tmp, lib)
    return lib


def build_torch_ops(force: bool = False, lib: Path = TORCH_OPS_LIB) -> Path:
    """The TORCH_LIBRARY(duplex_b200) ops (csrc/torch_ops.cpp) against torch's headers,
    linked to libduplex_b200.so (found next to it at run time)."""
    if (not force and lib.exists() and lib.stat().st_mtime > TORCH_OPS_SRC.stat().st_mtime
            and lib.stat().st_mtime > LIB.stat().st_mtime):
        return lib
    import torch
    from torch.utils import cpp_extension as ce
    abi = int(torch.compiled_with_cxx11_abi())
    cuda_inc = Path(nvcc_path()).resolve().parent.parent / "include"
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           str(TORCH_OPS_SRC), f"-I{INCLUDE}", f"-I{cuda_inc}"]
    cmd += [f"-I{p}" for p in ce.include_paths()]
    cmd += [f"-L{p}" for p in ce.library_paths()]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", f"-L{PKG}", "-lduplex_b200",
            "-Wl,-rpath,$ORIGIN", "-o", str(lib.with_suffix(".so.tmp"))]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("g++ failed on torch_ops.cpp:\n" + r.stdout + r.stderr)
    os.replace(lib.with_suffix(".so.tmp"), lib)
    return lib


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    build_torch_ops(force="--force" in sys.argv)
    print(LIB)
