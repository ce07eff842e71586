"""Loading of the native libraries (fails loudly when they are missing).

``load_ops()`` registers the ``rtdl_num_embeddings_cuda`` torch ops from
``_C.so``; ``capi()`` opens ``libple_b200.so`` with ctypes and declares the
C ABI of ``include/ple_capi.h``.  Both are built in-tree by
``python -m piecewiselinearembeddings_optimized_b200.build``.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libple_b200.so"
EXT_PATH = PKG / "_C.so"

_ops_loaded = False
_capi = None

# dtype codes and status codes of include/ple_capi.h
DTYPE_F32, DTYPE_F16, DTYPE_BF16, DTYPE_U8, DTYPE_I16, DTYPE_I32 = range(6)
EPILOGUE_NONE, EPILOGUE_A, EPILOGUE_B = range(3)
PLE_OK = 0


def _missing(path: Path) -> ImportError:
    return ImportError(
        f"native library {path.name} not found at {path}; build it with "
        "`python -m piecewiselinearembeddings_optimized_b200.build`"
    )


def load_ops():
    """Register the torch ops (idempotent) and return ``torch.ops.rtdl_num_embeddings_cuda``."""
    global _ops_loaded
    import torch

    if not _ops_loaded:
        for p in (LIB_PATH, EXT_PATH):
            if not p.exists():
                raise _missing(p)
        torch.ops.load_library(str(EXT_PATH))
        _ops_loaded = True
    return torch.ops.rtdl_num_embeddings_cuda


def capi() -> ctypes.CDLL:
    """The C ABI library with argument types declared."""
    global _capi
    if _capi is not None:
        return _capi
    if not LIB_PATH.exists():
        raise _missing(LIB_PATH)
    lib = ctypes.CDLL(str(LIB_PATH))
    P, I64, I, SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
    lib.ple_abi_version.restype = I
    lib.ple_abi_version.argtypes = []
    lib.ple_status_string.restype = ctypes.c_char_p
    lib.ple_status_string.argtypes = [I]
    lib.ple_last_error_message.restype = ctypes.c_char_p
    lib.ple_last_error_message.argtypes = []
    lib.ple_forward.restype = I
    lib.ple_forward.argtypes = [P, P, P, P, P, I64, I64, I64, I64, I, P, I, P, P]
    lib.ple_backward_workspace_size.restype = SZ
    lib.ple_backward_workspace_size.argtypes = [I64, I64, I64, I64]
    lib.ple_backward_kernel_kind.restype = I
    lib.ple_backward_kernel_kind.argtypes = [I64, I64, I64]
    lib.ple_backward.restype = I
    lib.ple_backward.argtypes = [P, I, P, P, P, P, P, P, I, I64, I64, I64, I64, P, P, P, SZ, P]
    lib.ple_embeddings_forward.restype = I
    lib.ple_embeddings_forward.argtypes = [P, P, P, P, P, P, P, P, I, I, I, I64, I64, I64, I64, I, P, I, P, P]
    lib.ple_embeddings_backward.restype = I
    lib.ple_embeddings_backward.argtypes = [P, I, P, P, P, P, P, P, P, P, I, I, I, I64, I64, I64, I64,
                                            P, I, P, P, P, P, P, P, SZ, P]
    lib.ple_embeddings_backward_noalloc.restype = I
    lib.ple_embeddings_backward_noalloc.argtypes = [P, I, P, P, P, P, P, P, P, P, I, I, I, I64, I64, I64, I64,
                                                    P, I, P, P, P, P, P, P]
    lib.ple_encoding_forward.restype = I
    lib.ple_encoding_forward.argtypes = [P, P, P, P, P, I, I64, I64, I64, I64, I, P, P]
    lib.ple_encoding_backward.restype = I
    lib.ple_encoding_backward.argtypes = [P, I, P, P, P, P, P, I, I64, I64, I64, I64, P, P]
    lib.ple_linear_status.restype = I
    lib.ple_linear_status.argtypes = []
    lib.ple_embeddings_linear_workspace_size.restype = SZ
    lib.ple_embeddings_linear_workspace_size.argtypes = [I64, I64, I64, I64, I]
    lib.ple_embeddings_linear_forward.restype = I
    lib.ple_embeddings_linear_forward.argtypes = [P, P, P, P, P, P, P, P, I, I, I, I64, I64, I64, I64,
                                                  P, I, P, I64, I, P, P, SZ, P]
    lib.ple_compute_bins.restype = I
    lib.ple_compute_bins.argtypes = [P, I64, I64, I, P, P, P, P]
    _capi = lib
    return lib


def check(status: int, what: str) -> None:
    if status != PLE_OK:
        lib = capi()
        raise RuntimeError(
            f"{what} failed: {lib.ple_status_string(status).decode()}: "
            f"{lib.ple_last_error_message().decode()}"
        )
