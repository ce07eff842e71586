"""Pointers for C-ABI calls that must be refused before anything is launched.

With a CUDA device present, every placeholder is the address of one real,
zeroed device buffer of ``BYTES`` bytes, larger than any tensor the refusal
tests declare (the largest is a 32 MiB weight).  A validation regression that
let such a call through would then launch on valid memory and show up as a
wrong status or wrong values, never as a device fault on a shared GPU.
Without a device the placeholder is a non-null address that no kernel can be
launched on.
"""
from __future__ import annotations

import ctypes

BYTES = 64 << 20
_buffer = None


def ptr() -> ctypes.c_void_p:
    global _buffer
    try:
        import torch

        if torch.cuda.is_available():
            if _buffer is None:
                _buffer = torch.zeros(BYTES, dtype=torch.uint8, device="cuda:0")
            return ctypes.c_void_p(_buffer.data_ptr())
    except ImportError:
        pass
    return ctypes.c_void_p(0x1000)
