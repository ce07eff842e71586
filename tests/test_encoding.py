"""Standalone piecewise-linear encoding (upstream ``PiecewiseLinearEncoding``):
the oracle's two formulations agree (CPU); the sm_100a kernels match the
oracle bit for bit in fp32 and after one rounding in bf16/fp16, in both
layouts, on the reference's bin cases plus edge ties, +-inf and NaN; the
gradient with respect to x matches the clamp rule (GPU)."""
from __future__ import annotations


import numpy as np
import pytest

from oracle import ple_oracle as o
from tests import cases

torch = pytest.importorskip("torch")


def _x_with_nan(bins, n, seed, integer=False):
    x = cases.sample_x(bins, n, seed, integer=integer, specials=True)
    x[5, :] = np.nan
    return x


# ---------------------------------------------------------------- CPU


@pytest.mark.parametrize("case", cases.BIN_CASES)
def test_oracle_layouts_agree_with_dense_encoding(case):
    bins = cases.make_bins(case)
    x = cases.sample_x(bins, 64, 11, integer=(case == "ties"))
    e, r, nb = o.pad_bins(bins)
    dense = o.dense_encoding(x, e, r, nb)
    padded = o.encoding(x, e, r, nb, padded=True, dtype=np.float64)
    np.testing.assert_array_equal(padded, dense)
    ragged = o.encoding(x, e, r, nb, dtype=np.float64)
    cols = np.concatenate([padded[:, i, [j if j < int(nb[i]) - 1 else e.shape[1] - 2 for j in range(int(nb[i]))]]
                           for i in range(len(bins))], axis=1)
    np.testing.assert_array_equal(ragged, cols)
    np.testing.assert_allclose(o.encoding(x, e, r, nb), ragged, rtol=1e-6, atol=1e-6)


def test_oracle_encoding_grad_matches_finite_differences():
    bins = cases.make_bins("ragged")
    x = cases.sample_x(bins, 32, 5).astype(np.float64)
    e, r, nb = o.pad_bins(bins)
    g = np.random.default_rng(2).standard_normal((32, int(nb.sum())))
    gx, _ = o.encoding_grad_x(g, x, e, r, nb)
    h = 1e-4
    fd = np.zeros_like(x)
    for i in range(x.shape[1]):
        xp, xm = x.copy(), x.copy()
        xp[:, i] += h
        xm[:, i] -= h
        fd[:, i] = ((o.encoding(xp, e, r, nb, dtype=np.float64) - o.encoding(xm, e, r, nb, dtype=np.float64))
                    * g).sum(1) / (2 * h)
    np.testing.assert_allclose(gx, fd, rtol=1e-3, atol=1e-3)


def test_encoding_fake_shapes():
    import rtdl_num_embeddings_cuda  # noqa: F401
    from torch._subclasses.fake_tensor import FakeTensorMode

    ops = torch.ops.rtdl_num_embeddings_cuda
    with FakeTensorMode():
        x = torch.empty(7, 3)
        e, r, n = torch.empty(3, 5), torch.empty(3, 4), torch.empty(3, dtype=torch.int32)
        off = torch.empty(4, dtype=torch.int64)
        assert ops.encoding_forward(x, e, r, n, off, 0, 10, torch.float32).shape == (7, 10)
        assert ops.encoding_forward(x, e, r, n, None, 1, 12, torch.bfloat16).shape == (7, 3, 4)
        assert ops.encoding_backward(torch.empty(7, 10), x, e, r, n, off, 0, 10).shape == (7, 3)


def test_encoding_module_construction_and_cpu_error():
    from rtdl_num_embeddings_cuda import CudaPiecewiseLinearEncoding

    bins = [torch.tensor(b) for b in cases.make_bins("ragged")]
    m = CudaPiecewiseLinearEncoding(bins)
    assert m.total_n_bins == sum(len(b) - 1 for b in bins)
    assert m._cuda_col_offsets.tolist()[-1] == m.total_n_bins
    assert dict(m.state_dict()) == {}
    from piecewiselinearembeddings_optimized_b200 import _compat

    if not _compat.HAVE_UPSTREAM:
        with pytest.raises(RuntimeError, match="no CPU implementation"):
            m(torch.zeros(2, len(bins)))
    with pytest.raises(ValueError):
        m(torch.zeros(2, len(bins) + 1))


def test_encoding_capi_rejects_bad_layouts():
    from piecewiselinearembeddings_optimized_b200 import _native

    lib = _native.capi()
    from tests import _placeholder

    fake = _placeholder.ptr()  # real device memory when a GPU is present; refused before any launch
    assert lib.ple_encoding_forward(fake, fake, fake, fake, fake, 7, 4, 3, 4, 12, 0, fake, None) == 1
    assert lib.ple_encoding_forward(fake, fake, fake, fake, fake, 1, 4, 3, 4, 11, 0, fake, None) == 2
    assert lib.ple_encoding_forward(fake, fake, fake, fake, None, 0, 4, 3, 4, 10, 0, fake, None) == 1
    assert lib.ple_encoding_backward(fake, 0, fake, fake, fake, fake, fake, 0, 4, 3, 4, 2, fake, None) == 2
    assert lib.ple_encoding_forward(None, fake, fake, fake, fake, 0, 0, 3, 4, 10, 0, None, None) == 0


# ---------------------------------------------------------------- GPU

TD = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _run(dev, bins, x, padded, out_mode, g=None):
    import rtdl_num_embeddings_cuda  # noqa: F401

    ops = torch.ops.rtdl_num_embeddings_cuda
    e, r, nb = o.pad_bins(bins)
    counts = [len(b) - 1 for b in bins]
    off = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    tx, te, tr, tn, toff = map(T, (x, e, r, nb, off))
    layout = 1 if padded else 0
    total = len(bins) * (e.shape[1] - 1) if padded else int(off[-1])
    y = ops.encoding_forward(tx, te, tr, tn, toff, layout, total, TD[out_mode])
    gx = None
    if g is not None:
        gx = ops.encoding_backward(T(g).to(TD[out_mode]), tx, te, tr, tn, toff, layout, total).cpu().numpy()
    return y.float().cpu().numpy(), gx


@pytest.mark.gpu
@pytest.mark.parametrize("case", cases.BIN_CASES)
@pytest.mark.parametrize("padded", [False, True])
@pytest.mark.parametrize("out_mode", ["f32", "bf16", "f16"])
def test_encoding_kernels_match_oracle(cuda_device, case, padded, out_mode):
    bins = cases.make_bins(case)
    x = _x_with_nan(bins, 256, 21, integer=(case == "ties"))
    e, r, nb = o.pad_bins(bins)
    ref = o.encoding(x, e, r, nb, padded=padded)
    g = np.random.default_rng(9).standard_normal(ref.shape).astype(np.float32)
    g = o.quantize(g, out_mode)
    y, gx = _run(cuda_device, bins, x, padded, out_mode, g)
    # fp32: same arithmetic as the oracle, bit for bit (NaN where the oracle has NaN); 16-bit: one rounding
    np.testing.assert_array_equal(y, o.quantize(ref, out_mode).astype(np.float32))
    ref_gx, ab = o.encoding_grad_x(g, x, e, r, nb, padded=padded)
    o.assert_reduction_close(gx, ref_gx, ab, rtol=1e-5, atol=1e-6, err_msg="grad_x")


@pytest.mark.gpu
@pytest.mark.parametrize("padded", [False, True])
def test_encoding_config_size(cuda_device, padded):
    """c2-sized batch (4096 x 64 features, up to 48 ragged bins)."""
    from piecewiselinearembeddings_optimized_b200 import workloads

    wl = workloads.make_workload("c2", n=4096)
    e, r, nb = o.pad_bins(wl.bins)
    ref = o.encoding(wl.x, e, r, nb, padded=padded)
    g = np.random.default_rng(4).standard_normal(ref.shape).astype(np.float32)
    y, gx = _run(cuda_device, wl.bins, wl.x, padded, "f32", g)
    np.testing.assert_array_equal(y, ref)
    ref_gx, ab = o.encoding_grad_x(g, wl.x, e, r, nb, padded=padded)
    o.assert_reduction_close(gx, ref_gx, ab, rtol=1e-5, atol=1e-6, err_msg="grad_x")


@pytest.mark.gpu
def test_encoding_module_autograd(cuda_device):
    from rtdl_num_embeddings_cuda import CudaPiecewiseLinearEncoding

    bins = cases.make_bins("wide")
    x = cases.sample_x(bins, 128, 3)
    m = CudaPiecewiseLinearEncoding([torch.from_numpy(b) for b in bins]).to(cuda_device)
    tx = torch.from_numpy(x).to(cuda_device).requires_grad_(True)
    y = m(tx)
    e, r, nb = o.pad_bins(bins)
    np.testing.assert_array_equal(y.detach().cpu().numpy(), o.encoding(x, e, r, nb))
    g = torch.randn_like(y)
    (y * g).sum().backward()
    ref_gx, ab = o.encoding_grad_x(g.cpu().numpy(), x, e, r, nb)
    o.assert_reduction_close(tx.grad.cpu().numpy(), ref_gx, ab, rtol=1e-5, atol=1e-6, err_msg="grad_x")
    # leading batch dimensions and the padded layout
    m.padded = True
    y3 = m(tx.detach().reshape(2, 64, -1))
    assert y3.shape == (2, 64, len(bins), e.shape[1] - 1)
