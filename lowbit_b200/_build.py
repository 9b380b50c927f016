"""Build of the CUDA library liblowbit_b200.so (sm_100a) from lowbit_b200/csrc.

The library is compiled in-tree with nvcc (one object per .cu, compiled in
parallel, linked with the static CUDA runtime) and loaded with ctypes. The
build output name does not change; a stamp file holding a hash of the sources
and flags decides whether a rebuild is needed.

Environment:
  NVCC               nvcc binary (default: $CUDA_HOME/bin/nvcc or nvcc on PATH)
  LOWBIT_B200_LIB    path to a prebuilt liblowbit_b200.so (skips the build)
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
LIB = PKG / "liblowbit_b200.so"
STAMP = PKG / ".liblowbit_b200.stamp"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# no fast-math: the activation quantizer relies on IEEE division and rint
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", "-diag-suppress", "177"]


def nvcc() -> str:
    env = os.environ.get("NVCC")
    if env:
        return env
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found; set NVCC or CUDA_HOME")
    return found


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _digest() -> str:
    h = hashlib.sha256()
    for p in sorted(list(CSRC.iterdir()) + list(INCLUDE.glob("*.h"))):
        if p.is_file() and p.suffix in (".cu", ".cuh", ".h"):
            h.update(p.name.encode())
            h.update(p.read_bytes())
    h.update(repr((ARCH, FLAGS)).encode())
    return h.hexdigest()[:16]


def up_to_date() -> bool:
    return LIB.exists() and STAMP.exists() and STAMP.read_text().strip() == _digest()


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile (if needed) and return the path of liblowbit_b200.so."""
    if os.environ.get("LOWBIT_B200_LIB"):
        return Path(os.environ["LOWBIT_B200_LIB"])
    if not force and up_to_date():
        return LIB
    cc = nvcc()
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)

    def compile_one(src: Path) -> Path:
        obj = objdir / (src.stem + ".o")
        cmd = [cc, *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        return obj

    with ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, *ARCH, "-shared", "-cudart", "static", *map(str, objs), "-o", str(tmp)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)  # atomic for concurrent importers
    STAMP.write_text(_digest())
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, force="--force" in sys.argv))
