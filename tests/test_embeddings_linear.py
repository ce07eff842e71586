"""The embeddings forward fused into the first Linear of its consumer
(``rtdl_num_embeddings_cuda::embeddings_linear_forward``, C ABI
``ple_embeddings_linear_forward``).

GPU: parity with the CPU oracle (bf16-autocast semantics: module output and
linear weight rounded to bf16, exact product) within one bf16 unit of the
embeddings; a tight check against this package's own embeddings kernel
followed by an exact float64 product (same bf16 embeddings, so only the fp32
accumulation of the tensor cores differs); shapes that exercise padding
features, partial row tiles, output widths that are not a multiple of 16,
two row sub-tiles, two MMAs per k-step and several column groups; the module
wrapper's forward and gradients against the unfused composition under
autocast.  CPU: workspace sizing and argument validation of the C ABI.
"""
from __future__ import annotations


import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import ple_oracle as o  # noqa: E402
from piecewiselinearembeddings_optimized_b200 import _native, workloads  # noqa: E402
from tests import _placeholder, cases  # noqa: E402

EPI = {"A": 1, "B": 2}
TORCH_DT = {"f32": torch.float32, "bf16": torch.bfloat16}
FAKE = None  # placeholder pointer for calls refused before any launch (set per test)


@pytest.fixture(autouse=True)
def _placeholder_pointer():
    """A real device buffer when a GPU is present (tests/_placeholder.py), else a non-null dummy."""
    global FAKE
    FAKE = _placeholder.ptr()


# ---------------------------------------------------------------- CPU: C ABI sizing and validation

def test_workspace_size_and_unsupported_shapes():
    lib = _native.capi()
    assert lib.ple_embeddings_linear_workspace_size(256, 32, 24, 256, _native.DTYPE_BF16) > 0
    assert lib.ple_embeddings_linear_workspace_size(512, 64, 16, 1000, _native.DTYPE_F32) > 0
    assert lib.ple_embeddings_linear_workspace_size(8, 16, 10, 64, _native.DTYPE_BF16) == 0  # D % 8 != 0
    assert lib.ple_embeddings_linear_workspace_size(8, 16, 16, 64, _native.DTYPE_F16) == 0
    assert lib.ple_embeddings_linear_workspace_size(8, 300, 16, 64, _native.DTYPE_BF16) == 0


def _call(lib, *, epi=1, bias="placeholder", compute=_native.DTYPE_BF16, wdt=_native.DTYPE_BF16,
          out=_native.DTYPE_F32, n=4, h=32):
    bias = FAKE if bias == "placeholder" else bias
    return lib.ple_embeddings_linear_forward(FAKE, FAKE, FAKE, FAKE, FAKE, bias, None, None, epi, 1, compute,
                                             n, 3, 4, 8, FAKE, wdt, None, h, out, FAKE, FAKE, 1 << 20, None)


def test_forward_rejects_bad_arguments():
    lib = _native.capi()
    assert _call(lib, compute=_native.DTYPE_F16) == 4
    assert _call(lib, wdt=_native.DTYPE_F32) == 4
    assert _call(lib, out=_native.DTYPE_F16) == 4
    assert _call(lib, bias=None) == 1 and b"bias" in lib.ple_last_error_message()
    assert _call(lib, h=0) == 2
    assert _call(lib, n=0) == 0  # empty batch: nothing to do


# ---------------------------------------------------------------- GPU parity

@pytest.fixture(scope="module")
def ops(cuda_device):
    import rtdl_num_embeddings_cuda  # noqa: F401

    return torch.ops.rtdl_num_embeddings_cuda


def _status():
    return _native.capi().ple_linear_status()


def _dev(dev, *arrays):
    return [None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in arrays]


def _problem(kind, n, d, h, version, seed):
    if kind in ("c4", "c5", "c3"):
        wl = workloads.make_workload(kind, n=n, f={"c4": 64, "c5": 32, "c3": 24}[kind], seed=seed)
        bins, x, d = wl.bins, wl.x, wl.d
    else:
        bins = cases.make_bins(kind)
        x = np.ascontiguousarray(cases.sample_x(bins, (n + 3) // 4 * 4, seed, integer=(kind == "ties"))[:n])
    edges, inv_w, nb = o.pad_bins(bins)
    w, bias, w0, b0 = cases.init_params(len(bins), edges.shape[1] - 1, d, version, seed)
    rng = np.random.default_rng(seed + 11)
    w1 = (rng.standard_normal((h, len(bins) * d)) / np.sqrt(len(bins) * d)).astype(np.float32)
    b1 = rng.uniform(-0.5, 0.5, h).astype(np.float32)
    return x, edges, inv_w, nb, w, bias, w0, b0, w1, b1


def _run(ops, dev, p, version, relu, mode, out_mode, with_b1=True):
    x, edges, inv_w, nb, w, bias, w0, b0, w1, b1 = p
    tx, te, tr, tn, tw, tb, tw0, tb0, tb1 = _dev(dev, x, edges, inv_w, nb, w, bias, w0, b0, b1 if with_b1 else None)
    tw1 = torch.from_numpy(w1).to(dev).to(torch.bfloat16)
    z = ops.embeddings_linear_forward(tx, te, tr, tn, tw, tb, tw0, tb0, EPI[version], relu, TORCH_DT[mode], tw1,
                                      tb1, TORCH_DT[out_mode])
    # this package's own embeddings kernel, rounded to bf16 as the A operand
    e = ops.embeddings_forward(tx, te, tr, tn, tw, tb, tw0, tb0, EPI[version], relu, TORCH_DT[mode], torch.bfloat16)
    torch.cuda.synchronize()
    return z.float().cpu().numpy(), e.float().cpu().numpy()


def _check(z, e_own, p, version, relu, mode, out_mode, with_b1=True):
    x, edges, inv_w, nb, w, bias, w0, b0, w1, b1 = p
    b1 = b1 if with_b1 else None
    z_ref, e_ref, scale = o.embeddings_linear_forward(x, edges, inv_w, nb, w, w1, b1, version=version,
                                                      activation=relu, bias=bias, w0=w0, b0=b0, mode=mode,
                                                      out_mode="f32")
    out_ulp = 2.0 ** -8 * np.abs(z_ref) if out_mode == "bf16" else 0.0
    # (1) the oracle: the embeddings may differ by one bf16 unit (epilogue B rounds x_ple once, the oracle twice)
    err = np.abs(z - z_ref)
    bound = 1e-2 * scale + 1e-3 + out_ulp
    assert np.all(err <= bound), f"max excess {np.max(err - bound)} (oracle)"
    np.testing.assert_allclose(e_own.reshape(e_ref.shape), e_ref, rtol=1e-2, atol=1e-2)
    # (2) own embeddings + exact product: only the tensor cores' fp32 accumulation differs
    n = e_own.shape[0]
    w1q = o.bf16_round(w1).astype(np.float64)
    z_own = e_own.reshape(n, -1).astype(np.float64) @ w1q.T + (0.0 if b1 is None else b1.astype(np.float64))
    scale_own = np.abs(e_own.reshape(n, -1).astype(np.float64)) @ np.abs(w1q).T
    err = np.abs(z - z_own)
    bound = 2e-3 * scale_own + 1e-5 + (2.0 ** -8 * np.abs(z_own) if out_mode == "bf16" else 0.0)
    assert np.all(err <= bound), f"max excess {np.max(err - bound)} (own embeddings, exact product)"


SHAPES = [
    # kind, n, d, h: padding features (F % G != 0), partial row tiles, H % 16 != 0, one or two row sub-tiles,
    # two MMAs per k-step (H > 256), several column groups (H > 512)
    ("ragged", 300, 8, 40),
    ("equal", 129, 16, 16),
    ("wide", 700, 24, 256),
    ("c4", 1024, None, 256),
    ("c5", 520, None, 384),
    ("c5", 260, None, 640),
    ("c3", 200, None, 96),
]


@pytest.mark.gpu
@pytest.mark.parametrize("kind,n,d,h", SHAPES)
@pytest.mark.parametrize("version", ["A", "B"])
@pytest.mark.parametrize("mode,out_mode", [("bf16", "bf16"), ("bf16", "f32"), ("f32", "f32")])
def test_matches_oracle_and_own_embeddings(ops, cuda_device, kind, n, d, h, version, mode, out_mode):
    relu = (n % 2 == 0) or version == "A"
    p = _problem(kind, n, d, h, version, 3)
    z, e = _run(ops, cuda_device, p, version, relu, mode, out_mode)
    assert z.shape == (n, h)
    assert _status() == 0
    _check(z, e, p, version, relu, mode, out_mode)


@pytest.mark.gpu
@pytest.mark.parametrize("case", cases.BIN_CASES)
def test_bin_cases_without_linear_bias(ops, cuda_device, case):
    p = _problem(case, 257, 16, 48, "B", 5)
    z, e = _run(ops, cuda_device, p, "B", True, "bf16", "f32", with_b1=False)
    assert _status() == 0
    _check(z, e, p, "B", True, "bf16", "f32", with_b1=False)


@pytest.mark.gpu
def test_deterministic_and_empty_batch(ops, cuda_device):
    p = _problem("c4", 600, None, 256, "B", 9)
    z1, _ = _run(ops, cuda_device, p, "B", True, "bf16", "f32")
    z2, _ = _run(ops, cuda_device, p, "B", True, "bf16", "f32")
    assert np.array_equal(z1, z2)
    x, edges, inv_w, nb, w, bias, w0, b0, w1, b1 = p
    tx, te, tr, tn, tw, tw0, tb0 = _dev(cuda_device, x[:0], edges, inv_w, nb, w, w0, b0)
    z = ops.embeddings_linear_forward(tx, te, tr, tn, tw, None, tw0, tb0, 2, True, torch.bfloat16,
                                      torch.from_numpy(w1).to(cuda_device).to(torch.bfloat16), None, torch.float32)
    assert tuple(z.shape) == (0, w1.shape[0])


@pytest.mark.gpu
def test_rejects_d_not_multiple_of_8(ops, cuda_device):
    p = _problem("equal", 64, 10, 32, "A", 1)
    with pytest.raises(RuntimeError, match="multiple of 8"):
        _run(ops, cuda_device, p, "A", True, "bf16", "f32")


# ---------------------------------------------------------------- module wrapper

def _modules(dev, version, d=16, h=96, seed=0):
    import rtdl_num_embeddings_cuda as rc

    torch.manual_seed(seed)
    bins = [torch.from_numpy(b) for b in workloads.make_workload("c5", n=8, f=24, seed=seed).bins]
    emb = rc.CudaPiecewiseLinearEmbeddings([b.to(dev) for b in bins], d, activation=True, version=version).to(dev)
    lin = torch.nn.Linear(len(bins) * d, h).to(dev)
    return emb, lin, rc.CudaPiecewiseLinearEmbeddingsLinear(emb, lin, fused=True)


@pytest.mark.gpu
@pytest.mark.parametrize("version", ["A", "B"])
def test_module_matches_composition_under_autocast(cuda_device, version):
    emb, lin, fused = _modules(cuda_device, version)
    x = torch.randn(333, emb.n_features, device=cuda_device)
    gz = torch.randn(333, lin.out_features, device=cuda_device)
    results = []
    for run in ("fused", "composition"):
        for p in list(emb.parameters()) + list(lin.parameters()):
            p.grad = None
        xr = x.clone().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            z = fused(xr) if run == "fused" else lin(emb(xr).flatten(1))
        assert z.dtype == torch.bfloat16
        z.float().backward(gz)
        grads = {n: p.grad.float().clone() for n, p in list(emb.named_parameters()) + list(lin.named_parameters())}
        grads["x"] = xr.grad.clone()
        results.append((z.float(), grads))
    (zf, gf), (zc, gc) = results
    torch.testing.assert_close(zf, zc, rtol=2e-2, atol=2e-2)
    for name in gc:
        ref = gc[name]
        tol = 2e-2 * float(ref.abs().max()) + 1e-3
        assert float((gf[name] - ref).abs().max()) <= tol, name
    assert _status() == 0


@pytest.mark.gpu
def test_module_bf16_linear_fp32_and_fallbacks(cuda_device):
    emb, lin, fused = _modules(cuda_device, "B")
    x = torch.randn(100, emb.n_features, device=cuda_device)
    with torch.no_grad():
        composed = lin(emb(x).flatten(1))
        assert torch.equal(fused(x), composed)  # plain fp32: the composition
        fused.bf16_linear = True
        z = fused(x)
        assert z.dtype == torch.float32
        e = emb(x).to(torch.bfloat16).double().flatten(1)
        ref = e @ lin.weight.to(torch.bfloat16).double().t() + lin.bias.double()
        scale = e.abs() @ lin.weight.to(torch.bfloat16).double().abs().t()
        assert bool(((z.double() - ref).abs() <= 2e-3 * scale + 1e-5).all())
        fused.fused = False  # the composition, whatever the dtypes
        assert torch.equal(fused(x), composed)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        assert torch.equal(fused(x), lin(emb(x).flatten(1)))


@pytest.mark.gpu
def test_module_more_than_256_bins_runs_the_composition(cuda_device):
    """The fused kernel's tables hold up to 256 bins; wider modules run the composition (bit-equal)."""
    import rtdl_num_embeddings_cuda as rc

    torch.manual_seed(4)
    rng = np.random.default_rng(4)
    bins = [torch.from_numpy((np.cumsum(rng.random(n + 1) + 0.01) - 0.3 * n).astype(np.float32))
            for n in (300, 9, 64)]
    emb = rc.CudaPiecewiseLinearEmbeddings([b.to(cuda_device) for b in bins], 16, activation=True,
                                           version="A").to(cuda_device)
    lin = torch.nn.Linear(len(bins) * 16, 32).to(cuda_device)
    fused = rc.CudaPiecewiseLinearEmbeddingsLinear(emb, lin, fused=True)
    x = torch.randn(64, len(bins), device=cuda_device) * 40
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        z = fused(x)
        assert z.dtype == torch.bfloat16
        assert torch.equal(z, lin(emb(x).flatten(1)))


@pytest.mark.gpu
def test_module_default_runs_the_composition(cuda_device):
    """Without fused=True the wrapper is exactly the composition (the fused kernel is opt-in: slower on the
    measured shapes), under autocast too."""
    import rtdl_num_embeddings_cuda as rc

    emb, lin, _ = _modules(cuda_device, "B")
    plain = rc.CudaPiecewiseLinearEmbeddingsLinear(emb, lin)
    assert plain.fused is False
    x = torch.randn(77, emb.n_features, device=cuda_device)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        assert torch.equal(plain(x), lin(emb(x).flatten(1)))
