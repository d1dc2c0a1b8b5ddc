"""Build the sm_100a kernels into the in-tree C-ABI library.

``python -m pymsst_b200.build`` compiles every ``csrc/*.cu`` with nvcc for
``sm_100a`` (objects under ``_build/``) and links
``pymsst_b200/_lib/libpymsst_b200.so``.  Objects are rebuilt only when a
source or header is newer.  nvcc cross-compiles, so this runs on a machine
without a GPU.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_DIR = PACKAGE_DIR.parent
CSRC_DIR = PACKAGE_DIR / "csrc"
INCLUDE_DIR = REPO_DIR / "include"
BUILD_DIR = REPO_DIR / "_build" / "pymsst_b200"
LIB_DIR = PACKAGE_DIR / "_lib"
LIB_PATH = LIB_DIR / "libpymsst_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-warn-spills",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.is_file():
        return str(candidate)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _sources() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))


def _newest_header_mtime() -> float:
    return max((p.stat().st_mtime for p in _headers()), default=0.0)


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD_DIR / (src.stem + ".o")
    if obj.is_file() and obj.stat().st_mtime >= max(src.stat().st_mtime, _newest_header_mtime()):
        return obj
    cmd = [_nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE_DIR), "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{result.stdout}\n{result.stderr}")
    if verbose and result.stderr.strip():
        print(result.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile and link the library; returns its path."""
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    sources = _sources()
    workers = jobs or min(len(sources), os.cpu_count() or 4)
    with ThreadPoolExecutor(max_workers=max(1, workers)) as pool:
        objects = list(pool.map(lambda s: _compile(s, verbose), sources))
    newest_obj = max(o.stat().st_mtime for o in objects)
    if LIB_PATH.is_file() and LIB_PATH.stat().st_mtime >= newest_obj:
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    # The CUDA runtime is linked statically; driver entry points (tensor-map
    # encoding) are resolved at run time, so the library loads without a GPU.
    cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objects)]
    if verbose:
        print(" ".join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"link failed:\n{result.stdout}\n{result.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    path = build(verbose="-v" in sys.argv)
    print(path)
