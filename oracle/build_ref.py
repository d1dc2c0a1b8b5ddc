"""Compile the reference's own CUDA extension into ``oracle/_ref/`` (checker only).

TEST INFRASTRUCTURE ONLY.  The reference (baicai-1145/pymsst) ships its fused
training kernels as two source files, src/pymsst/training/cuda/
fused_band_split.cpp and fused_band_split.cu, which its loader JIT-builds with
``torch.utils.cpp_extension.load`` (src/pymsst/training/fused_extension.py:45-55,
flags ``-O3 --use_fast_math`` and ``-lcublas``).  This recipe compiles the same
two files straight from the read-only reference tree with nvcc/g++ and the
same flags, adding the sm_100a target, and links a Python extension module
``oracle/_ref/pymsst_fused_band_split.so``.  Nothing is copied into this
repository.  The module is only imported by ``tests/golden/make_golden.py`` on
a GPU box to record golden vectors of the reference's kernels.

Usage: ``python oracle/build_ref.py --reference /path/to/pymsst`` (or the
checkout named by the PYMSST_REFERENCE environment variable).
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
MODULE = "pymsst_fused_band_split"


def reference_checkout(path: str | Path | None = None) -> Path | None:
    """The reference checkout: ``path`` if given, else $PYMSST_REFERENCE, else None."""
    if path:
        return Path(path)
    env = os.environ.get("PYMSST_REFERENCE")
    return Path(env) if env else None


def _torch_paths():
    import torch
    import torch.utils.cpp_extension as ce

    includes = ce.include_paths(device_type="cuda")
    libs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    return includes, libs, abi


def build(reference: str | Path | None = None, verbose: bool = False) -> Path | None:
    reference = reference_checkout(reference)
    if reference is None:
        if verbose:
            print("no reference checkout given (--reference or PYMSST_REFERENCE); skipping", file=sys.stderr)
        return None
    cuda_dir = reference / "src" / "pymsst" / "training" / "cuda"
    cpp = cuda_dir / "fused_band_split.cpp"
    cu = cuda_dir / "fused_band_split.cu"
    if not (cpp.is_file() and cu.is_file()):
        if verbose:
            print(f"reference sources not found under {cuda_dir}; skipping", file=sys.stderr)
        return None
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    target = OUT_DIR / f"{MODULE}.so"
    newest_src = max(cpp.stat().st_mtime, cu.stat().st_mtime, Path(__file__).stat().st_mtime)
    if target.is_file() and target.stat().st_mtime >= newest_src:
        return target

    includes, libs, abi = _torch_paths()
    py_include = sysconfig.get_paths()["include"]
    defines = [
        f"-DTORCH_EXTENSION_NAME={MODULE}",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
    ]
    inc = [f"-I{p}" for p in [*includes, py_include]]
    cu_obj = OUT_DIR / "fused_band_split.cu.o"
    cpp_obj = OUT_DIR / "fused_band_split.cpp.o"
    cmds = [
        [
            "/usr/local/cuda/bin/nvcc", "-c", str(cu), "-o", str(cu_obj), *defines, *inc,
            "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "--use_fast_math", "-std=c++17",
            "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
            "-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF_CONVERSIONS__",
            "-D__CUDA_NO_BFLOAT16_CONVERSIONS__", "-D__CUDA_NO_HALF2_OPERATORS__",
        ],
        ["g++", "-c", str(cpp), "-o", str(cpp_obj), *defines, *inc, "-O3", "-std=c++17", "-fPIC"],
        [
            "g++", "-shared", "-o", str(target), str(cu_obj), str(cpp_obj),
            *[f"-L{p}" for p in libs], *[f"-Wl,-rpath,{p}" for p in libs[:1]],
            "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
            "-lcudart", "-lcublas",
        ],
    ]
    for cmd in cmds:
        if verbose:
            print(" ".join(cmd), flush=True)
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"reference build step failed:\n{' '.join(cmd)}\n{result.stdout}\n{result.stderr}")
    for obj in (cu_obj, cpp_obj):
        obj.unlink(missing_ok=True)
    return target


def load(path: Path | None = None):
    """Import the compiled reference extension module (needs torch imported)."""
    import importlib.util

    import torch  # noqa: F401  (loads libtorch for the module's symbols)

    target = path or OUT_DIR / f"{MODULE}.so"
    spec = importlib.util.spec_from_file_location(MODULE, target)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


if __name__ == "__main__":
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference", type=Path, default=None)
    args = parser.parse_args()
    print(build(args.reference, verbose=True))
