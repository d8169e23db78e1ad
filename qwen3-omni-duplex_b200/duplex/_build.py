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


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
