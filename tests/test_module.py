"""The drop-in module ``rtdl_num_embeddings_cuda.CudaPiecewiseLinearEmbeddings``."""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import rtdl_num_embeddings_cuda as rnc  # noqa: E402
from oracle import ple_oracle as o  # noqa: E402
from tests import cases  # noqa: E402


def _bins(case="ragged"):
    return [torch.from_numpy(b) for b in cases.make_bins(case)]


def _init(m, seed):
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        m.linear.weight.copy_(torch.rand(m.linear.weight.shape, generator=g) * 0.2 + 0.05)
        if m.linear.bias is not None:
            m.linear.bias.copy_(torch.rand(m.linear.bias.shape, generator=g) * 0.2 + 0.1)
        if m.linear0 is not None:
            m.linear0.weight.copy_(torch.rand(m.linear0.weight.shape, generator=g) * 0.4 - 0.2)
            m.linear0.bias.copy_(torch.rand(m.linear0.bias.shape, generator=g) * 0.2 - 0.1)


# ---------------------------------------------------------------- CPU: construction and contract

@pytest.mark.parametrize("version", ["A", "B"])
def test_parameters_buffers_and_state_dict(version):
    bins = _bins()
    m = rnc.CudaPiecewiseLinearEmbeddings(bins, 12, activation=True, version=version)
    names = set(dict(m.named_parameters()))
    expect = {"linear.weight", "linear.bias"} if version == "A" else {"linear.weight", "linear0.weight",
                                                                      "linear0.bias"}
    assert names == expect
    assert set(m.state_dict()) == expect  # helper buffers are non-persistent
    assert m.linear.weight.shape == (4, 5, 12)
    assert m.get_output_shape() == torch.Size((4, 12))
    assert (m.n_features, m.max_n_bins, m.d_embedding) == (4, 5, 12)
    edges, inv_w, nb = o.pad_bins([b.numpy() for b in bins])
    np.testing.assert_array_equal(m._cuda_bin_edges.numpy(), edges)
    np.testing.assert_array_equal(m._cuda_inv_bin_widths.numpy(), inv_w)
    np.testing.assert_array_equal(m._cuda_n_bins.numpy(), nb)
    assert m._cuda_n_bins.dtype == torch.int32
    if version == "B":
        assert torch.count_nonzero(m.linear.weight) == 0  # PLE branch starts at zero


def test_state_dict_round_trip():
    a = rnc.CudaPiecewiseLinearEmbeddings(_bins(), 8, activation=False, version="B")
    b = rnc.CudaPiecewiseLinearEmbeddings(_bins(), 8, activation=False, version="B")
    _init(a, 1)
    b.load_state_dict(a.state_dict(), strict=True)
    for k, v in a.state_dict().items():
        assert torch.equal(v, b.state_dict()[k])


def test_constructor_errors():
    with pytest.raises(AssertionError):
        rnc.CudaPiecewiseLinearEmbeddings(_bins(), 65, activation=False, version="A")
    with pytest.raises(ValueError):
        rnc.CudaPiecewiseLinearEmbeddings([torch.tensor([1.0, 0.0])], 8, activation=False, version="A")
    with pytest.raises(ValueError):
        rnc.CudaPiecewiseLinearEmbeddings([torch.tensor([0.0])], 8, activation=False, version="A")
    with pytest.warns(UserWarning):
        m = rnc.CudaPiecewiseLinearEmbeddings(_bins(), 8, activation=False)
    assert m.linear.bias is not None  # version None behaves as "A"


def test_input_validation_on_cpu():
    m = rnc.CudaPiecewiseLinearEmbeddings(_bins(), 8, activation=False, version="A")
    with pytest.raises(ValueError):
        m(torch.zeros(3))
    with pytest.raises(ValueError):
        m(torch.zeros(3, 5))
    with pytest.raises(RuntimeError):  # no CPU compute path in this package
        m(torch.zeros(3, 4))


def test_fake_tensor_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    ops = torch.ops.rtdl_num_embeddings_cuda
    with FakeTensorMode():
        x = torch.empty(5, 4, device="cuda")
        e = torch.empty(4, 6, device="cuda")
        r = torch.empty(4, 5, device="cuda")
        n = torch.empty(4, dtype=torch.int32, device="cuda")
        w = torch.empty(4, 5, 8, device="cuda")
        y, idx = ops.forward(x, e, r, n, w, torch.bfloat16)
        assert y.shape == (5, 4, 8) and y.dtype == torch.bfloat16 and idx.dtype == torch.uint8
        y2 = ops.embeddings_forward(x, e, r, n, w, None, None, None, 0, False, torch.float32, torch.float32)
        assert y2.shape == (5, 4, 8)
        gx, gw, gb, gw0, gb0 = ops.embeddings_backward(y2, x, e, r, n, w, None, None, None, None, 0, False,
                                                       torch.float32, True, True, True, True)
        assert gx.shape == (5, 4) and gw.shape == (4, 5, 8) and gb.numel() == 0


# ---------------------------------------------------------------- GPU: autograd through the module

@pytest.mark.gpu
@pytest.mark.parametrize("version", ["A", "B"])
@pytest.mark.parametrize("activation", [False, True])
@pytest.mark.parametrize("case", ["equal", "ragged", "single_bin", "all_single_bin", "ties"])
def test_module_autograd_matches_oracle(cuda_device, version, activation, case):
    _check_module_autograd(cuda_device, _bins(case), version, activation, integer=(case == "ties"))


@pytest.mark.gpu
@pytest.mark.parametrize("version", ["A", "B"])
@pytest.mark.parametrize("activation", [False, True])
def test_module_autograd_more_than_256_bins(cuda_device, version, activation):
    """300 bins in one feature: int16 bin indices and the wide-bin kernels, through the module and autograd."""
    rng = np.random.default_rng(17)
    bins = [torch.from_numpy((np.cumsum(rng.random(n + 1) + 0.01) - 0.3 * n).astype(np.float32))
            for n in (300, 4, 1, 57)]
    _check_module_autograd(cuda_device, bins, version, activation)


def _check_module_autograd(cuda_device, bins, version, activation, integer=False):
    m = rnc.CudaPiecewiseLinearEmbeddings(bins, 16, activation=activation, version=version).to(cuda_device)
    _init(m, 3)
    xn = cases.sample_x([b.numpy() for b in bins], 128, 5, integer=integer)
    x = torch.from_numpy(xn).to(cuda_device).requires_grad_(True)
    y = m(x)
    assert y.dtype == torch.float32 and y.shape == (128, len(bins), 16)
    gn = np.random.default_rng(2).standard_normal(tuple(y.shape)).astype(np.float32)
    y.backward(torch.from_numpy(gn).to(cuda_device))
    edges, inv_w, nb = o.pad_bins([b.numpy() for b in bins])
    p = {k: v.detach().cpu().numpy() for k, v in m.named_parameters()}
    kw = dict(version=version, activation=activation, bias=p.get("linear.bias"), w0=p.get("linear0.weight"),
              b0=p.get("linear0.bias"))
    y_ref, _, _ = o.embeddings_forward(xn, edges, inv_w, nb, p["linear.weight"], **kw)
    np.testing.assert_allclose(y.detach().cpu().numpy(), y_ref, rtol=1e-5, atol=1e-6)
    ref = o.embeddings_backward(gn, xn, edges, inv_w, nb, p["linear.weight"], **kw)
    tol = dict(rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(x.grad.cpu().numpy(), ref["grad_x"], **tol)
    o.assert_reduction_close(m.linear.weight.grad.cpu().numpy(), ref["grad_W"], ref["abs"]["grad_W"], **tol)
    if version == "A":
        o.assert_reduction_close(m.linear.bias.grad.cpu().numpy(), ref["grad_bias"], ref["abs"]["grad_bias"], **tol)
    else:
        o.assert_reduction_close(m.linear0.weight.grad.cpu().numpy(), ref["grad_w0"], ref["abs"]["grad_w0"], **tol)
        o.assert_reduction_close(m.linear0.bias.grad.cpu().numpy(), ref["grad_b0"], ref["abs"]["grad_b0"], **tol)


@pytest.mark.gpu
@pytest.mark.parametrize("version", ["A", "B"])
def test_module_autocast_bf16(cuda_device, version):
    bins = _bins("ragged")
    m = rnc.CudaPiecewiseLinearEmbeddings(bins, 16, activation=True, version=version).to(cuda_device)
    _init(m, 4)
    xn = cases.sample_x([b.numpy() for b in bins], 128, 6)
    x = torch.from_numpy(xn).to(cuda_device).requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = m(x)
    assert y.dtype == torch.float32  # fp32 epilogue promotes, as in the reference
    gn = o.bf16_round(np.random.default_rng(1).standard_normal(tuple(y.shape)).astype(np.float32))
    y.backward(torch.from_numpy(gn).to(cuda_device))
    assert m.linear.weight.grad.dtype == torch.float32 and x.grad.dtype == torch.float32
    edges, inv_w, nb = o.pad_bins([b.numpy() for b in bins])
    p = {k: v.detach().cpu().numpy() for k, v in m.named_parameters()}
    kw = dict(version=version, activation=True, bias=p.get("linear.bias"), w0=p.get("linear0.weight"),
              b0=p.get("linear0.bias"), mode="bf16")
    y_ref, _, _ = o.embeddings_forward(xn, edges, inv_w, nb, p["linear.weight"], **kw)
    np.testing.assert_allclose(y.detach().cpu().numpy(), y_ref, rtol=1e-2, atol=1e-2)
    ref = o.embeddings_backward(gn, xn, edges, inv_w, nb, p["linear.weight"], **kw)
    np.testing.assert_allclose(x.grad.cpu().numpy(), ref["grad_x"], rtol=2e-2, atol=2e-2)
    np.testing.assert_allclose(m.linear.weight.grad.cpu().numpy(), ref["grad_W"], rtol=2e-2, atol=2e-2)


@pytest.mark.gpu
def test_module_errors_on_cuda(cuda_device):
    m = rnc.CudaPiecewiseLinearEmbeddings(_bins(), 8, activation=False, version="A").to(cuda_device)
    with pytest.raises(TypeError):
        m(torch.zeros(4, 4, dtype=torch.float64, device=cuda_device))
    with pytest.raises(ValueError):
        m(torch.zeros(4, 8, device=cuda_device)[:, ::2])
    with pytest.raises(TypeError):  # float64 parameters are rejected like the reference's
        m.double()(torch.zeros(4, 4, device=cuda_device))


@pytest.mark.gpu
def test_torch_compile_fullgraph(cuda_device):
    bins = _bins("equal")
    m = rnc.CudaPiecewiseLinearEmbeddings(bins, 8, activation=True, version="B").to(cuda_device)
    _init(m, 7)
    x = torch.from_numpy(cases.sample_x([b.numpy() for b in bins], 64, 3)).to(cuda_device)
    eager = m(x)
    compiled = torch.compile(m, fullgraph=True, dynamic=True)
    out = compiled(x)
    torch.testing.assert_close(out, eager, rtol=0, atol=0)
    xg = x.clone().requires_grad_(True)
    compiled(xg).sum().backward()
    xe = x.clone().requires_grad_(True)
    m(xe).sum().backward()
    torch.testing.assert_close(xg.grad, xe.grad, rtol=0, atol=0)
