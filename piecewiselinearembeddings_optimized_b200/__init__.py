"""B200-native piecewise-linear embeddings (sm_100a).

The drop-in Python surface is the ``rtdl_num_embeddings_cuda`` package at the
repository root (same module, class, op names and semantics as the
reference).  This package holds the CUDA kernels and C-ABI library
(``csrc/``), the build step (``build.py``), the native loader
(``_native.py``), the host-side mirror of the reference interface
(``module.py``, ``_meta.py``, ``_autograd.py``) and the data-parallel helper
(``parallel.py``).

Importing this package loads no native code; ``ops()`` / the module class do,
and raise if the CUDA library is missing.
"""

__version__ = "0.1.0"
