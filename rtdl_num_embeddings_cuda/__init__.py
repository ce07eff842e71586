"""Drop-in replacement for the reference package ``rtdl_num_embeddings_cuda``.

Same import contract as the reference (``__init__.py:5-8``): loading the
package registers the ``rtdl_num_embeddings_cuda`` torch ops (native
library), then their fake and autograd registrations, then exposes
``CudaPiecewiseLinearEmbeddings``.  The implementation lives in
``piecewiselinearembeddings_optimized_b200`` (sm_100a kernels behind a C ABI).
"""
from piecewiselinearembeddings_optimized_b200 import _native

_native.load_ops()
from piecewiselinearembeddings_optimized_b200 import _meta as _meta  # noqa: E402,F401
from piecewiselinearembeddings_optimized_b200 import _autograd as _autograd  # noqa: E402,F401
from piecewiselinearembeddings_optimized_b200.module import (  # noqa: E402
    CudaPiecewiseLinearEmbeddings,
    CudaPiecewiseLinearEmbeddingsLinear,
    CudaPiecewiseLinearEncoding,
)

from piecewiselinearembeddings_optimized_b200.bins import bin_tables, compute_bins  # noqa: E402

__all__ = ["CudaPiecewiseLinearEmbeddings", "CudaPiecewiseLinearEmbeddingsLinear", "CudaPiecewiseLinearEncoding",
           "compute_bins", "bin_tables"]

__version__ = "0.2.0.dev0+b200"
