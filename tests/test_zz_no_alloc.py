"""ple_embeddings_backward_noalloc: the fused backward with the library's
built-in scratch instead of a caller workspace, for callers that cannot hand
over device memory of their own (plain C FFI hosts without a device
allocator, serving processes that reserve all memory at start-up).

Its results must equal those of ple_embeddings_backward on two calls in a
row, and again after calls of the same and of another shape have left
garbage (NaN partial sums) in the shared scratch: every scratch slot the backward reads must be
written earlier in the same call.  The main kernels are deterministic, so
their results are compared bitwise; the wide-bin path (more than 256 bins)
sums grad_W with atomics (any order) and is compared within the parity tests'
summation-order bound (rtol 1e-4, atol 1e-5 plus 2^-20 of the sum of the
terms' magnitudes), its other gradients within rtol 1e-4, atol 1e-5.  The refusal of shapes beyond the scratch needs
no device and is a CPU test in test_capi.py.  The file name sorts last so that
these tests also run after every other GPU test in the same process.
"""
from __future__ import annotations

import numpy as np
import pytest

from piecewiselinearembeddings_optimized_b200 import _native

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 16 << 20
GRAD_NAMES = ("grad_x", "grad_W", "grad_bias", "grad_w0", "grad_b0")


def _inputs(torch, dev, name, n, f):
    from oracle import ple_oracle as o
    from piecewiselinearembeddings_optimized_b200 import workloads

    wl = workloads.make_workload(name, n=n, f=f)
    edges, inv_w, nb = o.pad_bins(wl.bins)
    T = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    gdt = torch.bfloat16 if wl.out_mode == "bf16" else torch.float32
    g = T(workloads.make_grad(wl)).to(gdt)
    return wl, g, [T(a) for a in (wl.x, edges, inv_w, nb, wl.weight, wl.bias, wl.w0, wl.b0)]


class _Call:
    """Argument lists of one backward configuration for both entry points."""

    def __init__(self, torch, dev, wl, g, tensors, epi, relu):
        self.torch, self.dev, self.wl, self.g = torch, dev, wl, g
        self.x, self.e, self.r, self.nb, self.w, self.bias, self.w0, self.b0 = tensors
        self.epi, self.relu = epi, relu
        self.code = {torch.float32: 0, torch.bfloat16: 2}[g.dtype]
        self.qcode = 2 if wl.mode == "bf16" else 0
        self.shape = (wl.n, wl.f, wl.max_n_bins, wl.d)

    def head(self, g=None):
        P = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        g = self.g if g is None else g
        return (P(g), self.code, P(self.x), P(self.e), P(self.r), P(self.nb), P(self.w), P(self.bias), P(self.w0),
                P(self.b0), self.epi, self.relu, self.qcode, *self.shape, None, 3)

    def grads(self):
        n, f, b, d = self.shape
        return [self.torch.full(s, float("nan"), device=self.dev) for s in ((n, f), (f, b, d), (f, d), (f, d), (f, d))]

    def wanted(self, name):
        return ((name != "grad_bias" or self.epi == 1) and (name not in ("grad_w0", "grad_b0") or self.epi == 2))


def _run_reference(lib, c, stream):
    ws_bytes = lib.ple_backward_workspace_size(*c.shape)
    ws = c.torch.empty(ws_bytes, dtype=c.torch.uint8, device=c.dev)
    out = c.grads()
    _native.check(lib.ple_embeddings_backward(*c.head(), *[t.data_ptr() for t in out], ws.data_ptr(), ws_bytes,
                                              stream), "ple_embeddings_backward")
    return out


def _run_noalloc(lib, c, stream, g=None):
    out = c.grads()
    _native.check(lib.ple_embeddings_backward_noalloc(*c.head(g), *[t.data_ptr() for t in out], stream),
                  "ple_embeddings_backward_noalloc")
    return out


def _compare(torch, c, ref, got, exact, what, bounds=None):
    from oracle import ple_oracle as o

    for name, a, b in zip(GRAD_NAMES, ref, got):
        if not c.wanted(name):
            continue
        if exact:
            assert torch.equal(a, b), f"{what}: {name} differs from ple_embeddings_backward"
        elif name in bounds:  # sums in atomic order: within the summation-order bound of the parity tests
            o.assert_reduction_close(b.cpu().numpy(), a.cpu().numpy(), bounds[name], err_msg=f"{what}: {name}")
        else:
            torch.testing.assert_close(b, a, rtol=1e-4, atol=1e-5, msg=f"{what}: {name}")


CASES = [  # name, n, f, epilogue, relu, exact
    ("c1", 1000, None, None, None, True),
    ("c2", 4096, 32, None, None, True),
    ("c4", 8192, 64, None, None, True),
    ("wide", 512, 3, 0, 0, False),  # 300 bins, bare x_ple op: the wide-bin kernels
]


@pytest.mark.parametrize("name,n,f,epi,relu,exact", CASES, ids=[c[0] for c in CASES])
def test_noalloc_matches_workspace_entry_point(cuda_device, name, n, f, epi, relu, exact):
    import torch

    lib = _native.capi()
    stream = torch.cuda.current_stream().cuda_stream
    if name == "wide":
        from oracle import ple_oracle as o
        from tests import cases

        rng = np.random.default_rng(5)
        # ragged wide features (300, 5 and 120 bins): cumulative sums of seeded steps, as the parity tests
        bins = [(np.cumsum(rng.random(k + 1) + 0.01) - 0.3 * k).astype(np.float32) for k in (300, 5, 120)][:f]
        wl_x = cases.sample_x(bins, n, 12)
        edges, inv_w, nb = o.pad_bins(bins)
        B = edges.shape[1] - 1
        W = rng.uniform(0.05, 0.25, (f, B, 8)).astype(np.float32)
        T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_device)  # noqa: E731

        class _WL:
            pass

        wl = _WL()
        wl.n, wl.f, wl.max_n_bins, wl.d, wl.mode = n, f, B, 8, "f32"
        g = T(rng.standard_normal((n, f, 8)).astype(np.float32))
        c = _Call(torch, cuda_device, wl, g, [T(a) for a in (wl_x, edges, inv_w, nb, W)] + [None, None, None],
                  epi, relu)
        # 2 x sum of |terms| of each grad_W element: |g| times the largest |t| of the feature's samples
        gn = g.cpu().numpy()
        k = o.bin_index(wl_x, edges, nb)
        tmax = np.maximum(1.0, np.abs(o.position(wl_x, k, edges, inv_w)).max(axis=0))
        bounds = {"grad_W": np.broadcast_to((np.abs(gn).sum(0) * tmax[:, None])[:, None, :], (f, B, 8)) * 2}
    else:
        wl, g, tensors = _inputs(torch, cuda_device, name, n, f)
        c = _Call(torch, cuda_device, wl, g, tensors, 2 if wl.version == "B" else 1, int(wl.activation))
        bounds = {}
    assert lib.ple_backward_workspace_size(*c.shape) <= SCRATCH_BYTES
    ref = _run_reference(lib, c, stream)
    # two calls in a row
    for call in range(2):
        got = _run_noalloc(lib, c, stream)
        torch.cuda.synchronize()
        _compare(torch, c, ref, got, exact, f"call {call}", bounds)
    # garbage in the shared scratch: NaN partial sums from a call of the same shape (exactly the slots the
    # checked call uses) and from a call of another shape, both with a NaN upstream gradient
    _run_noalloc(lib, c, stream, g=torch.full_like(c.g, float("nan")))
    other_wl, other_g, other_t = _inputs(torch, cuda_device, "c1", 777, 5)
    other = _Call(torch, cuda_device, other_wl, other_g.fill_(float("nan")), other_t, 2, 1)
    _run_noalloc(lib, other, stream)
    got = _run_noalloc(lib, c, stream)
    torch.cuda.synchronize()
    _compare(torch, c, ref, got, exact, "after NaN calls of the same and of another shape", bounds)
