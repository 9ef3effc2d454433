"""Build libsva_b200.so in-tree with nvcc for sm_100a.

Usage: ``python -m sva_b200.build`` (or ``__graft_entry__.build()``).  The shared library is
written next to this file so that it travels with the source tree; nothing is installed.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "libsva_b200.so"
SOURCES = ["capi.cu", "catalog.cu", "decode.cu", "postings.cu", "inverted.cu", "adapter.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "--shared",
    "-Xptxas", "-O3",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libsva_b200.so")
    return cand


def sources() -> list[Path]:
    return [CSRC / s for s in SOURCES if (CSRC / s).exists()]


def needs_build() -> bool:
    if not OUT.exists():
        return True
    mtime = OUT.stat().st_mtime
    deps = sources() + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [HERE.parent / "include" / "sva_b200.h"]
    return any(d.stat().st_mtime > mtime for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every source to an object in parallel (one nvcc per file), then link the library."""
    if not force and not needs_build():
        return OUT
    from concurrent.futures import ThreadPoolExecutor

    objdir = HERE / "_build"
    objdir.mkdir(exist_ok=True)
    nvcc = nvcc_path()
    compile_flags = [f for f in NVCC_FLAGS if f != "--shared"]

    def compile_one(src: Path) -> tuple[Path, subprocess.CompletedProcess]:
        obj = objdir / (src.stem + ".o")
        cmd = [nvcc, *compile_flags, "-I", str(HERE.parent / "include"), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        return obj, subprocess.run(cmd, capture_output=True, text=True)

    with ThreadPoolExecutor(max_workers=len(sources())) as pool:
        results = list(pool.map(compile_one, sources()))
    for obj, res in results:
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {obj.stem}.cu ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "--shared", "-Xcompiler", "-fPIC",
           *[str(o) for o, _ in results], "-o", str(tmp), "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
