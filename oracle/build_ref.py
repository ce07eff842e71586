"""Compile the reference's own CUDA ops from their sources into ``oracle/_ref/``.

TEST INFRASTRUCTURE ONLY: the resulting library is the *reference* (used to
produce golden vectors that pin the CPU oracle), never the product.

The reference path is three source files, ``csrc/ops.cpp``,
``csrc/forward_cuda.cu`` and ``csrc/backward_cuda.cu`` (+ ``common.cuh``),
which compile directly with nvcc/g++ against torch's headers; the reference's
own build system (``setup.py``) is not used.  Outputs go only to
``oracle/_ref/``; nothing is copied into the repository.

The library registers the op namespace ``rtdl_num_embeddings_cuda`` - the
same namespace as the product - so it must be loaded in a separate process
(``tests/golden/make_golden.py`` and ``oracle/time_reference_cuda.py`` do that).

Usage: ``python oracle/build_ref.py [--reference DIR]``.  The reference
project is found at ``--reference``, else at ``$PLE_REFERENCE_DIR``, else in a
directory named ``reference`` beside this repository.  A no-op when the
reference sources are absent (e.g. on a GPU box, which uses the prebuilt
file).
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
LIB = OUT_DIR / "rtdl_ref_ops.so"


def default_reference() -> Path:
    """$PLE_REFERENCE_DIR, else a directory named ``reference`` beside this repository."""
    env = os.environ.get("PLE_REFERENCE_DIR")
    return Path(env) if env else HERE.parent.parent / "reference"


def _torch_paths():
    import torch
    from torch.utils import cpp_extension

    inc = cpp_extension.include_paths()
    libdir = cpp_extension.library_paths()[0]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    return inc, libdir, abi


def build(reference: Path | None = None, force: bool = False) -> Path | None:
    csrc = (reference or default_reference()) / "csrc"
    sources = [csrc / "ops.cpp", csrc / "forward_cuda.cu", csrc / "backward_cuda.cu"]
    if not all(s.exists() for s in sources):
        return LIB if LIB.exists() else None
    newest = max(s.stat().st_mtime for s in sources + [csrc / "common.cuh"])
    if LIB.exists() and not force and LIB.stat().st_mtime > newest:
        return LIB
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    inc, libdir, abi = _torch_paths()
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    py_inc = sysconfig.get_paths()["include"]
    defs = [
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        "-DTORCH_EXTENSION_NAME=rtdl_ref_ops",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
    ]
    incs = [f"-I{p}" for p in inc] + [f"-I{py_inc}", f"-I{csrc}"]
    objs = []
    for src in sources:
        obj = OUT_DIR / (src.stem + ".o")
        if src.suffix == ".cu":
            cmd = [
                f"{cuda_home}/bin/nvcc", "-c", str(src), "-o", str(obj),
                "-gencode", "arch=compute_100a,code=sm_100a",
                "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
                "-Xcompiler", "-fPIC",
                "-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF_CONVERSIONS__",
                "-D__CUDA_NO_BFLOAT16_CONVERSIONS__", "-D__CUDA_NO_HALF2_OPERATORS__",
            ] + defs + incs
        else:
            cmd = ["g++", "-c", str(src), "-o", str(obj), "-O2", "-std=c++17", "-fPIC",
                   f"-I{cuda_home}/include"] + defs + incs
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    link = ["g++", "-shared", "-o", str(LIB)] + objs + [
        f"-L{libdir}", f"-Wl,-rpath,{libdir}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
        "-ltorch_cuda", f"-L{cuda_home}/lib64", "-lcudart",
    ]
    subprocess.run(link, check=True)
    for o in objs:
        Path(o).unlink()
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=None)
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    lib = build(args.reference, args.force)
    print(lib if lib else "reference sources absent; nothing built")
    return 0


if __name__ == "__main__":
    sys.exit(main())
