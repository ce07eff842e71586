"""Build the native libraries in-tree for sm_100a.

* ``libple_b200.so`` - the CUDA kernels and the C ABI (``include/ple_capi.h``),
  compiled with nvcc for ``-gencode arch=compute_100a,code=sm_100a`` and
  linked with the static CUDA runtime; no torch dependency.
* ``_C.so`` - the torch adapter (``csrc/ops.cpp``): registers the
  ``rtdl_num_embeddings_cuda`` ops and calls the C ABI; loaded with
  ``torch.ops.load_library``.

Usage: ``python -m piecewiselinearembeddings_optimized_b200.build [--force]``.
Objects go to ``_build/`` next to this file; the libraries next to this file.
Rebuilds only what is older than its sources.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
BUILD = PKG / "_build"
LIB = PKG / "libple_b200.so"
EXT = PKG / "_C.so"

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              f"-I{INCLUDE}", f"-I{CSRC}"]


def _newer(target: Path, deps) -> bool:
    if not target.exists():
        return False
    t = target.stat().st_mtime
    return all(Path(d).stat().st_mtime <= t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r


def build_capi(force: bool = False, verbose: bool = False) -> Path:
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE / "ple_capi.h"]
    BUILD.mkdir(exist_ok=True)
    objs = [BUILD / (s.stem + ".o") for s in sources]
    todo = [(s, o) for s, o in zip(sources, objs) if force or not _newer(o, [s] + headers)]

    def compile_one(so):
        s, o = so
        cmd = [f"{CUDA_HOME}/bin/nvcc", "-c", str(s), "-o", str(o)] + ARCH + NVCC_FLAGS
        if verbose:
            cmd += ["-Xptxas", "-v"]
        r = _run(cmd)
        if verbose:
            (BUILD / (s.stem + ".ptxas.txt")).write_text(r.stderr)

    with ThreadPoolExecutor(max_workers=max(1, min(len(todo), os.cpu_count() or 4))) as ex:
        list(ex.map(compile_one, todo))
    if force or todo or not _newer(LIB, objs):
        _run([f"{CUDA_HOME}/bin/nvcc", "-shared", "-o", str(LIB)] + [str(o) for o in objs] + ARCH +
             ["-cudart", "static"])
    return LIB


def build_ext(force: bool = False) -> Path:
    src = CSRC / "ops.cpp"
    if not force and _newer(EXT, [src, INCLUDE / "ple_capi.h", LIB]):
        return EXT
    import torch
    from torch.utils import cpp_extension

    inc = cpp_extension.include_paths()
    libdir = cpp_extension.library_paths()[0]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-shared", "-fPIC", "-O2", "-std=c++17", str(src), "-o", str(EXT),
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", f"-I{INCLUDE}", f"-I{CUDA_HOME}/include"]
    cmd += [f"-I{p}" for p in inc]
    cmd += [f"-L{PKG}", "-lple_b200", "-Wl,-rpath,$ORIGIN",
            f"-L{libdir}", f"-Wl,-rpath,{libdir}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu"]
    _run(cmd)
    return EXT


def build(force: bool = False, verbose: bool = False) -> None:
    build_capi(force, verbose)
    build_ext(force)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="keep ptxas -v output in _build/")
    args = ap.parse_args(argv)
    build(args.force, args.verbose)
    print(LIB)
    print(EXT)
    return 0


if __name__ == "__main__":
    sys.exit(main())
