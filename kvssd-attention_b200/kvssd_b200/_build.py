"""Builds libkvssd_b200.so from ``csrc/`` with nvcc for sm_100a, in-tree.

The library is a plain C-ABI shared object (no torch headers, no Python extension module):
``python -m kvssd_b200._build`` or ``kvssd_b200._build.build()`` compiles every ``csrc/*.cu``
and ``csrc/*.cpp`` (host-only code) into ``kvssd_b200/lib/libkvssd_b200.so``. Objects are rebuilt only when a source or header
is newer than the library.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
ROOT_DIR = PACKAGE_DIR.parent
CSRC_DIR = ROOT_DIR / "csrc"
INCLUDE_DIR = ROOT_DIR.parent / "include"
LIB_DIR = PACKAGE_DIR / "lib"
LIB_PATH = LIB_DIR / "libkvssd_b200.so"
BUILD_DIR = ROOT_DIR / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH_FLAGS,
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _sources() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cu")) + sorted(CSRC_DIR.glob("*.cpp"))


def _headers() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(dep.stat().st_mtime > mtime for dep in deps)


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compiles the CUDA sources and links the shared library; returns its path."""
    nvcc = _nvcc()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    headers = _headers()
    jobs = []
    objects = []
    for src in _sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objects.append(obj)
        if force or _stale(obj, [src, *headers]):
            extra = ["-Xcompiler", "-pthread"] if src.suffix == ".cpp" else []
            cmd = [nvcc, *NVCC_FLAGS, *extra, "-I", str(INCLUDE_DIR), "-c", str(src), "-o", str(obj)]
            jobs.append(cmd)

    def run(cmd: list[str]) -> None:
        if verbose:
            print(" ".join(cmd), flush=True)
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        list(pool.map(run, jobs))
    if force or jobs or _stale(LIB_PATH, objects):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        run([nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objects), "-lpthread"])
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    path = build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(path)
