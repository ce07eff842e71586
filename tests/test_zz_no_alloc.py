"""ple_embeddings_backward_noalloc: the fused backward with the library's
built-in scratch instead of a caller workspace.  Its results must equal those
of ple_embeddings_backward (same kernels, deterministic) on two calls in a
row, and shapes whose workspace exceeds the scratch must be refused before
any launch.  The file name sorts last so that the test also runs after every
other GPU test in the same process."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from piecewiselinearembeddings_optimized_b200 import _native

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 16 << 20
PLE_ERR_WORKSPACE = 5


def _inputs(torch, dev, name, n, f):
    from oracle import ple_oracle as o
    from piecewiselinearembeddings_optimized_b200 import workloads

    wl = workloads.make_workload(name, n=n, f=f)
    edges, inv_w, nb = o.pad_bins(wl.bins)
    T = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    gdt = torch.bfloat16 if wl.out_mode == "bf16" else torch.float32
    g = T(workloads.make_grad(wl)).to(gdt)
    return wl, g, [T(a) for a in (wl.x, edges, inv_w, nb, wl.weight, wl.bias, wl.w0, wl.b0)]


def _grads(torch, dev, wl):
    f, b, d = wl.f, wl.max_n_bins, wl.d
    return [torch.full(s, float("nan"), device=dev) for s in ((wl.n, f), (f, b, d), (f, d), (f, d), (f, d))]


@pytest.mark.parametrize("name,n,f", [("c1", 1000, None), ("c2", 4096, 32), ("c4", 8192, 64)])
def test_noalloc_matches_workspace_entry_point_twice(cuda_device, name, n, f):
    import torch

    lib = _native.capi()
    wl, g, (x, e, r, nb, w, bias, w0, b0) = _inputs(torch, cuda_device, name, n, f)
    P = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    code = {torch.float32: 0, torch.bfloat16: 2}
    gcode = code[g.dtype]
    qcode = 2 if wl.mode == "bf16" else 0
    epi = 2 if wl.version == "B" else 1
    F, B, D = wl.f, wl.max_n_bins, wl.d
    assert lib.ple_backward_workspace_size(wl.n, F, B, D) <= SCRATCH_BYTES
    stream = torch.cuda.current_stream().cuda_stream

    def head():
        return (P(g), gcode, P(x), P(e), P(r), P(nb), P(w), P(bias), P(w0), P(b0), epi, int(wl.activation), qcode,
                wl.n, F, B, D, None, 3)

    ws_bytes = lib.ple_backward_workspace_size(wl.n, F, B, D)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda_device)
    ref = _grads(torch, cuda_device, wl)
    _native.check(lib.ple_embeddings_backward(*head(), *[P(t) for t in ref], P(ws), ws_bytes, stream),
                  "ple_embeddings_backward")
    for call in range(2):
        got = _grads(torch, cuda_device, wl)
        _native.check(lib.ple_embeddings_backward_noalloc(*head(), *[P(t) for t in got], stream),
                      "ple_embeddings_backward_noalloc")
        torch.cuda.synchronize()
        for name_, a, b in zip(("grad_x", "grad_W", "grad_bias", "grad_w0", "grad_b0"), ref, got):
            wanted = (name_ != "grad_bias" or epi == 1) and (name_ not in ("grad_w0", "grad_b0") or epi == 2)
            if wanted:
                assert torch.equal(a, b), f"call {call}: {name_} differs from ple_embeddings_backward"


def test_noalloc_refuses_shapes_beyond_the_scratch(cuda_device):
    import torch

    lib = _native.capi()
    # many small feature chunks per CTA range give many partial slots; the first plannable shape above the scratch
    for n, f, b, d in ((64, 1024, 256, 32), (256, 8192, 128, 32), (1 << 20, 8192, 64, 64)):
        need = lib.ple_backward_workspace_size(n, f, b, d)
        if need > SCRATCH_BYTES:
            break
    assert need > SCRATCH_BYTES
    fake = ctypes.c_void_p(0x1000)  # never dereferenced: the size check runs before any device access
    st = lib.ple_embeddings_backward_noalloc(fake, 0, fake, fake, fake, fake, fake, None, None, None, 0, 0, 0,
                                             n, f, b, d, None, 3, fake, fake, None, None, None, None)
    assert st == PLE_ERR_WORKSPACE
    msg = lib.ple_last_error_message().decode()
    assert str(need) in msg and "ple_embeddings_backward" in msg
    torch.cuda.synchronize()
