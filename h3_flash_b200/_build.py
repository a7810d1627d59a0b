"""Builds libh3b.so (the sm_100a kernels behind include/h3b.h) in-tree with nvcc.

The library is a plain C-ABI shared object: each ``csrc/*.cu`` is compiled for
``sm_100a`` only and linked with the static CUDA runtime, so the ``.so`` that
travels with the source tree needs nothing but the NVIDIA driver at run time.
"""

from __future__ import annotations

import concurrent.futures
import fcntl
import os
import shutil
import subprocess
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = PACKAGE_DIR.parent / "include"
LIB_DIR = PACKAGE_DIR / "lib"
LIB_PATH = LIB_DIR / "libh3b.so"
OBJ_DIR = PACKAGE_DIR.parent / "_build" / "obj"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
    *ARCH_FLAGS,
]


def nvcc_path() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
    return found


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    inputs = _sources() + _headers() + [Path(__file__)]
    return any(path.stat().st_mtime > built for path in inputs)


def _compile(nvcc: str, source: Path, extra: list[str], verbose: bool) -> Path:
    obj = OBJ_DIR / (source.stem + ".o")
    cmd = [nvcc, *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(source), "-o", str(obj)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or result.returncode != 0:
        print(" ".join(cmd))
        print(result.stdout, result.stderr)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed on {source.name}:\n{result.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile every csrc/*.cu for sm_100a and link lib/libh3b.so. Returns its path."""

    if not force and not is_stale():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    # Processes started together (one per GPU) build once: the others wait on
    # the lock and then find the library fresh.
    with open(LIB_DIR / ".build.lock", "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        if not force and not is_stale():
            return LIB_PATH
        return _build_locked(verbose, ptxas_verbose)


def _build_locked(verbose: bool, ptxas_verbose: bool) -> Path:
    nvcc = nvcc_path()
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    sources = _sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(sources))) as pool:
        objects = list(pool.map(lambda s: _compile(nvcc, s, extra, verbose), sources))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objects)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"link failed:\n{result.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    import sys

    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv,
                ptxas_verbose="--ptxas" in sys.argv))
