"""The C ABI library: exports, host-side validation (CPU) and direct calls (GPU)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from piecewiselinearembeddings_optimized_b200 import _native
from tests import _placeholder

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions():
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names.update(re.findall(r"\b(ple_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    names = declared_functions()
    assert len(names) >= 8
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_abi_version_and_status_strings():
    lib = _native.capi()
    hdr = (ROOT / "include" / "ple_capi.h").read_text()
    ver = int(re.search(r"#define PLE_ABI_VERSION (\d+)", hdr).group(1))
    assert lib.ple_abi_version() == ver
    assert lib.ple_status_string(0) == b"ok"
    assert lib.ple_status_string(2) == b"invalid shape"
    assert lib.ple_status_string(99) == b"unknown status"


def test_backward_kernel_kind_without_a_device():
    """Kernel choice from the sizes alone (B200 defaults when no device is visible): the histogram kernel for
    d_embedding 8 / 16 / 24 up to 256 bins, the sorted kernel for other widths, the wide kernels above 256 bins,
    a negative status for refused sizes."""
    import os

    lib = _native.capi()
    hist = 0 if os.environ.get("PLE_BACKWARD_KERNEL") == "sorted" else 1
    assert lib.ple_backward_kernel_kind(512, 64, 16) == hist
    assert lib.ple_backward_kernel_kind(256, 32, 24) == hist
    assert lib.ple_backward_kernel_kind(8, 16, 8) == hist
    assert lib.ple_backward_kernel_kind(512, 64, 32) == 0
    assert lib.ple_backward_kernel_kind(128, 64, 64) == 0
    assert lib.ple_backward_kernel_kind(3, 10, 15) == 0
    assert lib.ple_backward_kernel_kind(4, 1000, 16) == 2
    assert lib.ple_backward_kernel_kind(0, 16, 16) < 0
    assert lib.ple_backward_kernel_kind(4, 16, 0) < 0


FAKE = None  # placeholder pointer for calls refused before any launch (set per test)


@pytest.fixture(autouse=True)
def _placeholder_pointer():
    """A real device buffer when a GPU is present (tests/_placeholder.py), else a non-null dummy."""
    global FAKE
    FAKE = _placeholder.ptr()


@pytest.mark.parametrize("n,f,b,d,code,msg", [
    (4, 0, 4, 8, 2, "n_features"),
    (4, 3, 0, 8, 2, "max_n_bins"),
    (4, 3, 4, 0, 2, "d_embedding"),
    (-1, 3, 4, 8, 2, "batch"),
    (4, 3, 4, 65, 4, "<= 64"),
    (4, 3, (1 << 20) + 1, 8, 4, "max_n_bins"),
])
def test_forward_rejects_bad_sizes(n, f, b, d, code, msg):
    lib = _native.capi()
    st = lib.ple_forward(FAKE, FAKE, FAKE, FAKE, FAKE, n, f, b, d, 0, FAKE, 3, None, None)
    assert st == code
    assert msg in lib.ple_last_error_message().decode()


def test_wide_bins_only_for_the_bare_op():
    """More than 256 bins: the bare x_ple op runs its wide-bin kernels; an
    epilogue or activation is refused before any launch."""
    lib = _native.capi()
    st = lib.ple_embeddings_forward(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, None, None, 1, 0, 0,
                                    4, 3, 300, 8, 0, FAKE, 3, None, None)
    assert st == 4 and b"max_n_bins > 256" in lib.ple_last_error_message()
    st = lib.ple_embeddings_forward(FAKE, FAKE, FAKE, FAKE, FAKE, None, None, None, 0, 1, 0,
                                    4, 3, 300, 8, 0, FAKE, 3, None, None)
    assert st == 4
    # grad_output, dtype, x, edges, inv_w, n_bins, W, bias, w0, b0, epilogue A, relu, compute, N, F, B, D,
    # bin_indices, dtype, grad_x, grad_W, grad_bias, grad_w0, grad_b0, workspace, bytes, stream
    st = lib.ple_embeddings_backward(FAKE, 0, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, None, None, 1, 1, 0,
                                     4, 3, 300, 8, None, 0, FAKE, FAKE, FAKE, None, None, FAKE, 1 << 20, None)
    assert st == 4 and b"max_n_bins > 256" in lib.ple_last_error_message()
    assert lib.ple_backward_workspace_size(4, 3, 300, 8) == 2 * 3 * 300 * 8 * 4
    assert lib.ple_backward_workspace_size(4, 3, (1 << 20) + 1, 8) == 0


def test_forward_rejects_missing_tables_and_bad_dtypes():
    lib = _native.capi()
    assert lib.ple_forward(FAKE, None, FAKE, FAKE, FAKE, 4, 3, 4, 8, 0, FAKE, 3, None, None) == 1
    assert lib.ple_forward(FAKE, FAKE, FAKE, FAKE, FAKE, 4, 3, 4, 8, 7, FAKE, 3, None, None) == 1
    assert lib.ple_forward(FAKE, FAKE, FAKE, FAKE, FAKE, 4, 3, 4, 8, 0, FAKE, 0, FAKE, None) == 1
    st = lib.ple_embeddings_forward(FAKE, FAKE, FAKE, FAKE, FAKE, None, None, None, 1, 0, 0,
                                    4, 3, 4, 8, 0, FAKE, 3, None, None)
    assert st == 1 and b"bias" in lib.ple_last_error_message()
    st = lib.ple_embeddings_forward(FAKE, FAKE, FAKE, FAKE, FAKE, None, FAKE, None, 2, 0, 0,
                                    4, 3, 4, 8, 0, FAKE, 3, None, None)
    assert st == 1 and b"w0" in lib.ple_last_error_message()


def test_empty_batch_forward_is_a_no_op():
    lib = _native.capi()
    assert lib.ple_forward(None, FAKE, FAKE, FAKE, FAKE, 0, 3, 4, 8, 0, None, 3, None, None) == 0


def test_backward_requires_workspace_before_any_launch():
    lib = _native.capi()
    st = lib.ple_backward(FAKE, 0, FAKE, FAKE, FAKE, FAKE, FAKE, None, 3, 4, 3, 4, 8, FAKE, FAKE,
                          None, 0, None)
    assert st == 5


NOALLOC_SCRATCH_BYTES = 16 << 20


def test_noalloc_refuses_shapes_beyond_the_scratch():
    """ple_embeddings_backward_noalloc refuses a shape whose workspace exceeds its
    built-in scratch, before any launch, naming the size and the entry point to use."""
    lib = _native.capi()
    # many small features: more than 16 MiB of partial sums whatever the device properties
    for n, f, b, d in ((64, 1 << 20, 16, 8), (64, 1024, 256, 32), (256, 8192, 128, 32)):
        need = lib.ple_backward_workspace_size(n, f, b, d)
        if need > NOALLOC_SCRATCH_BYTES:
            break
    assert need > NOALLOC_SCRATCH_BYTES
    st = lib.ple_embeddings_backward_noalloc(FAKE, 0, FAKE, FAKE, FAKE, FAKE, FAKE, None, None, None, 0, 0, 0,
                                             n, f, b, d, None, 3, FAKE, FAKE, None, None, None, None)
    assert st == 5
    msg = lib.ple_last_error_message().decode()
    assert str(need) in msg and "ple_embeddings_backward" in msg
    # more than 256 bins: accepted for the bare op (the wide-bin kernels) but refused with an epilogue
    st = lib.ple_embeddings_backward_noalloc(FAKE, 0, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, None, None, 1, 1, 0,
                                             4, 3, 300, 8, None, 3, FAKE, FAKE, FAKE, None, None, None)
    assert st == 4 and b"max_n_bins > 256" in lib.ple_last_error_message()


# ---------------------------------------------------------------- GPU: direct calls


@pytest.mark.gpu
def test_direct_capi_forward_backward_match_oracle(cuda_device):
    import torch

    from oracle import ple_oracle as o
    from tests import cases

    lib = _native.capi()
    bins = cases.make_bins("ragged")
    x = cases.sample_x(bins, 256, 11)
    edges, inv_w, nb = o.pad_bins(bins)
    f, b, d = len(bins), edges.shape[1] - 1, 16
    w, _, w0, b0 = cases.init_params(f, b, d, "B", 5)
    g = np.random.default_rng(4).standard_normal((256, f, d)).astype(np.float32)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_device)  # noqa: E731
    tx, te, tr, tn, tw, tw0, tb0, tg = map(T, (x, edges, inv_w, nb, w, w0, b0, g))
    out = torch.empty(256, f, d, device=cuda_device)
    idx = torch.empty(256, f, dtype=torch.uint8, device=cuda_device)
    stream = torch.cuda.current_stream().cuda_stream
    _native.check(lib.ple_forward(tx.data_ptr(), te.data_ptr(), tr.data_ptr(), tn.data_ptr(), tw.data_ptr(),
                                  256, f, b, d, 0, out.data_ptr(), 3, idx.data_ptr(), stream), "ple_forward")
    y = out.cpu().numpy()
    xp, k = o.x_ple_forward(x, edges, inv_w, nb, w)
    np.testing.assert_array_equal(idx.cpu().numpy(), k)
    np.testing.assert_allclose(y, xp, rtol=1e-5, atol=1e-6)

    ws_bytes = lib.ple_backward_workspace_size(256, f, b, d)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda_device)
    gx = torch.empty(256, f, device=cuda_device)
    gw = torch.empty(f, b, d, device=cuda_device)
    gw0 = torch.empty(f, d, device=cuda_device)
    gb0 = torch.empty(f, d, device=cuda_device)
    _native.check(lib.ple_embeddings_backward(
        tg.data_ptr(), 0, tx.data_ptr(), te.data_ptr(), tr.data_ptr(), tn.data_ptr(), tw.data_ptr(), None,
        tw0.data_ptr(), tb0.data_ptr(), 2, 1, 0, 256, f, b, d, idx.data_ptr(), 3, gx.data_ptr(), gw.data_ptr(),
        None, gw0.data_ptr(), gb0.data_ptr(), ws.data_ptr(), ws_bytes, stream), "ple_embeddings_backward")
    ref = o.embeddings_backward(g, x, edges, inv_w, nb, w, version="B", activation=True, w0=w0, b0=b0)
    np.testing.assert_allclose(gx.cpu().numpy(), ref["grad_x"], rtol=1e-4, atol=1e-5)
    for got, key in ((gw, "grad_W"), (gw0, "grad_w0"), (gb0, "grad_b0")):
        o.assert_reduction_close(got.cpu().numpy(), ref[key], ref["abs"][key], err_msg=key)


@pytest.mark.gpu
def test_backward_rejects_small_workspace(cuda_device):
    import torch

    lib = _native.capi()
    t = torch.zeros(64, device=cuda_device)
    nb = torch.ones(3, dtype=torch.int32, device=cuda_device)
    ws = torch.empty(16, dtype=torch.uint8, device=cuda_device)
    st = lib.ple_backward(t.data_ptr(), 0, t.data_ptr(), t.data_ptr(), t.data_ptr(), nb.data_ptr(), t.data_ptr(),
                          None, 3, 4, 3, 2, 4, t.data_ptr(), t.data_ptr(), ws.data_ptr(), 16, None)
    assert st == 5
    torch.cuda.synchronize()
