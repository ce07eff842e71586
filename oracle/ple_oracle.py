"""CPU restatement of the reference PLE path (TEST INFRASTRUCTURE ONLY).

This module is the oracle the CUDA path is checked against. It is never
imported by the product package; only tests, ``__graft_entry__.smoke()`` and
the CPU-baseline leg of ``bench.py`` may use it.

Two independent formulations live here:

* the *pairwise* restatement of the reference kernels
  (``csrc/forward_cuda.cu``, ``csrc/backward_cuda.cu``, ``csrc/common.cuh``):
  right-sided bin search, extrapolating position, logical-to-physical bin
  map, left-to-right fp32 prefix, ``fma(t, W[phys k], prefix)``, and the
  closed-form gradients including the ``x == e_k`` boundary sub-gradient;
* the *dense* formulation of the third-party dependency the reference
  subclasses, ``rtdl_num_embeddings==0.0.12`` (``pyproject.toml:17``;
  not vendored in the reference): a clamped ``[N, F, B]`` encoding with
  ragged masking contracted with ``weight[F, B, D]``.  It is written from the
  published algorithm (Gorishniy et al., "On Embeddings for Numerical
  Features in Tabular Deep Learning", piecewise-linear encoding, eq. 1) and is
  used as an independent cross-check and as the CPU baseline.

Pinning: ``tests/test_oracle.py`` checks the pairwise restatement
against golden vectors produced by the reference's own CUDA ops
(``tests/golden/make_golden.py``, compiled from the reference sources by
``oracle/build_ref.py``).

All arrays are numpy; values that live in a reduced-precision dtype on the
GPU (bf16/fp16) are carried here as float32 arrays holding exactly the
rounded values.
"""
from __future__ import annotations

import numpy as np

VERSIONS = ("A", "B")
MODES = ("f32", "bf16", "f16")


# ---------------------------------------------------------------------------
# Rounding helpers (common.cuh:81-96, quantize_to_float<T>)
# ---------------------------------------------------------------------------

def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    bits = a.view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000
    out = rounded.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(a), a, out).astype(np.float32)


def quantize(a: np.ndarray, mode: str) -> np.ndarray:
    """Round through the mode's storage type and back to float32.

    Follows ``quantize_to_float<scalar_t>`` (common.cuh:81-96): the reference
    emulates autocast's low-precision matmul inputs by rounding W and the
    position to the output type before the fp32 FMA.
    """
    a = np.asarray(a, dtype=np.float32)
    if mode == "f32":
        return a
    if mode == "bf16":
        return bf16_round(a)
    if mode == "f16":
        with np.errstate(over="ignore"):
            return a.astype(np.float16).astype(np.float32)
    raise ValueError(f"unknown mode {mode!r}")


def fma32(a: np.ndarray, b: np.ndarray, c: np.ndarray) -> np.ndarray:
    """fp32 fused multiply-add emulated in float64 (product exact, one rounding)."""
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(
        np.float32
    )


# ---------------------------------------------------------------------------
# Module construction helpers (module.py:58-131)
# ---------------------------------------------------------------------------

def pad_bins(bins: list[np.ndarray]):
    """Padded edge table, fp32 reciprocal widths and real bin counts.

    Follows ``CudaPiecewiseLinearEmbeddings.__init__`` (module.py:58-109):
    edges are padded with +inf to ``[F, B+1]``; ``inv_bin_widths[F, B]`` holds
    ``reciprocal(e[1:] - e[:-1])`` computed in fp32 and zero in the padding;
    ``n_bins`` is int32.
    """
    n_bins = np.array([len(b) - 1 for b in bins], dtype=np.int32)
    if (n_bins < 1).any():
        raise ValueError("every feature needs at least two edges")
    f, bmax = len(bins), int(n_bins.max())
    edges = np.full((f, bmax + 1), np.inf, dtype=np.float32)
    inv_w = np.zeros((f, bmax), dtype=np.float32)
    for i, b in enumerate(bins):
        e = np.asarray(b, dtype=np.float32)
        edges[i, : e.size] = e
        with np.errstate(divide="ignore"):
            inv_w[i, : e.size - 1] = (np.float32(1.0) / (e[1:] - e[:-1])).astype(np.float32)
    return edges, inv_w, n_bins


def bin_indices_dtype(max_n_bins: int):
    """Storage type of the saved bin index (``_meta.py:14-19``)."""
    if max_n_bins <= 256:
        return np.uint8
    if max_n_bins <= 32768:
        return np.int16
    return np.int32


# ---------------------------------------------------------------------------
# Pairwise restatement of the reference kernels
# ---------------------------------------------------------------------------

def bin_index(x: np.ndarray, edges: np.ndarray, n_bins: np.ndarray) -> np.ndarray:
    """Logical bin of every (sample, feature) pair.

    ``k = clamp(searchsorted(e[0..n], x, right) - 1, 0, n - 1)``; NaN compares
    false with every edge and lands in the last real bin
    (``find_logical_bin_right``, common.cuh:27-63).
    """
    x = np.asarray(x, dtype=np.float32)
    n, f = x.shape
    k = np.empty((n, f), dtype=np.int64)
    for i in range(f):
        nb = int(n_bins[i])
        e = edges[i, : nb + 1]
        # count of edges e_j with !(x < e_j); NaN counts every edge.
        cnt = np.searchsorted(e, x[:, i], side="right")
        cnt = np.where(np.isnan(x[:, i]), nb + 1, cnt)
        k[:, i] = np.clip(cnt - 1, 0, nb - 1)
    return k


def physical_bin(k: np.ndarray, n_real: np.ndarray, max_n_bins: int) -> np.ndarray:
    """Last real bin is stored at column ``B - 1`` (common.cuh:66-78)."""
    return np.where(k == n_real - 1, max_n_bins - 1, k)


def position(x, k, edges, inv_w):
    """Unclamped position ``t = (x - e_k) * r_k`` in fp32 (forward_cuda.cu:223-225)."""
    f_idx = np.arange(x.shape[1])[None, :]
    e_k = edges[f_idx, k]
    r_k = inv_w[f_idx, k]
    return ((np.asarray(x, np.float32) - e_k).astype(np.float32) * r_k).astype(np.float32)


def prefix_tables(W: np.ndarray, n_bins: np.ndarray, mode: str):
    """Per-feature tables in logical-bin order.

    ``P[i, k, :] = sum_{j<k} q(W[i, j, :])`` accumulated left to right in fp32
    (forward_cuda.cu:135-176, one thread per D component adding bins in
    order) and ``S[i, k, :] = q(W[i, phys(k), :])``.
    """
    f, b, d = W.shape
    Wq = quantize(W, mode)
    P = np.zeros((f, b, d), dtype=np.float32)
    S = np.zeros((f, b, d), dtype=np.float32)
    for i in range(f):
        nb = int(n_bins[i])
        acc = np.zeros(d, dtype=np.float32)
        for j in range(nb):
            P[i, j] = acc
            phys = b - 1 if j == nb - 1 else j
            S[i, j] = Wq[i, phys]
            acc = (acc + Wq[i, phys]).astype(np.float32)
    return P, S


def x_ple_forward(x, edges, inv_w, n_bins, W, mode: str = "f32"):
    """``x_ple[b, i, :] = sum_{j<k} W[i, j] + t * W[i, phys(k)]``.

    Restates ``ple_forward_shared_kernel`` (forward_cuda.cu:20-290): the
    prefix comes from ``prefix_tables``, the active row is combined with
    ``fmaf(q(t), q(W[phys k]), prefix)`` and the result is rounded to the
    output type (``static_cast<output_t>``, forward_cuda.cu:270-281).
    Returns ``(x_ple, k)`` with ``x_ple`` a float32 array of rounded values.
    """
    x = np.asarray(x, dtype=np.float32)
    k = bin_index(x, edges, n_bins)
    t = position(x, k, edges, inv_w)
    P, S = prefix_tables(W, n_bins, mode)
    f_idx = np.arange(x.shape[1])[None, :]
    pre = P[f_idx, k]          # [N, F, D]
    slope = S[f_idx, k]        # [N, F, D]
    tq = quantize(t, mode)[..., None]
    out = fma32(tq, slope, pre)
    return quantize(out, mode), k


def x_ple_backward(g, x, edges, inv_w, n_bins, W, mode: str = "f32", with_abs: bool = False):
    """Gradients of ``x_ple`` with respect to ``x`` and ``weight``.

    * ``grad_x = r_k <g, q(W[phys k])> + [k>0 and x == e_k] r_{k-1} <g, q(W[k-1])>``
      (``ple_backward_grad_x_kernel``, backward_cuda.cu:343-492; the second
      term is the inclusive clamp sub-gradient at an interior edge);
    * ``grad_W[i, phys(j)] = sum_{k_b = j} q(t_b) g_b + sum_{k_b > j} g_b`` for
      ``j < n_i`` and zero in padding rows (reverse prefix over bins,
      backward_cuda.cu:268-336 and 859-925).

    Sums are accumulated in float64.  With ``with_abs`` a third result holds
    the same reduction over absolute values (``sum |terms|`` per grad_W
    element), the scale of any fp32 summation error.
    """
    x = np.asarray(x, dtype=np.float32)
    g = np.asarray(g, dtype=np.float32)
    n, f = x.shape
    b_max, d = W.shape[1], W.shape[2]
    k = bin_index(x, edges, n_bins)
    t = position(x, k, edges, inv_w)
    tq = quantize(t, mode).astype(np.float64)
    Wq = quantize(W, mode).astype(np.float64)
    g64 = g.astype(np.float64)
    f_idx = np.arange(f)[None, :]
    phys = physical_bin(k, n_bins[None, :], b_max)
    r_k = inv_w[f_idx, k].astype(np.float64)
    dot_k = np.einsum("nfd,nfd->nf", g64, Wq[f_idx, phys])
    grad_x = r_k * dot_k
    e_k = edges[f_idx, k]
    boundary = (k > 0) & (x == e_k)
    if boundary.any():
        km1 = np.maximum(k - 1, 0)
        r_prev = inv_w[f_idx, km1].astype(np.float64)
        dot_prev = np.einsum("nfd,nfd->nf", g64, Wq[f_idx, km1])
        grad_x = grad_x + np.where(boundary, r_prev * dot_prev, 0.0)

    grad_W = _reverse_prefix(k, tq, g64, n_bins, f, b_max, d)
    if with_abs:
        return grad_x, grad_W, _reverse_prefix(k, np.abs(tq), np.abs(g64), n_bins, f, b_max, d)
    return grad_x, grad_W


def _reverse_prefix(k, tq, g64, n_bins, f, b_max, d):
    """``grad_W[i, phys(j)] = U[j] + sum_{j'>j} H[j']`` (zero padding rows)."""
    grad_W = np.zeros((f, b_max, d), dtype=np.float64)
    for i in range(f):
        nb = int(n_bins[i])
        ki = k[:, i]
        H = np.zeros((nb, d))
        U = np.zeros((nb, d))
        np.add.at(H, ki, g64[:, i, :])
        np.add.at(U, ki, tq[:, i, None] * g64[:, i, :])
        suffix = np.zeros(d)
        for j in range(nb - 1, -1, -1):
            phys_j = b_max - 1 if j == nb - 1 else j
            grad_W[i, phys_j] = U[j] + suffix
            suffix = suffix + H[j]
    return grad_W


# ---------------------------------------------------------------------------
# Module-level composition (module.py:207-248) and its autograd
# ---------------------------------------------------------------------------

def linear0(x, w0, b0):
    """Version-B per-feature affine term ``x * w0 + b0`` ([F, D] weight and bias)."""
    return fma32(np.asarray(x, np.float32)[..., None], w0[None], b0[None])


def embeddings_forward(x, edges, inv_w, n_bins, W, *, version="A", activation=False,
                       bias=None, w0=None, b0=None, mode="f32", out_mode="f32"):
    """Forward of ``CudaPiecewiseLinearEmbeddings`` (module.py:207-248).

    ``y = [x*w0 + b0] + act(x_ple + [bias])``. Under autocast (``mode`` bf16 or
    f16) ``x_ple`` is produced in the low-precision type and the bias, ReLU and
    linear0 add run in fp32 (type promotion with the fp32 parameters);
    ``out_mode`` is the storage type of the final result.
    Returns ``(y, z, k)``: output, pre-activation ``x_ple + bias`` and bins.
    """
    xp, k = x_ple_forward(x, edges, inv_w, n_bins, W, mode)
    z = xp
    if version == "A" and bias is not None:
        z = (z + bias[None]).astype(np.float32)
    y = np.maximum(z, np.float32(0.0)) if activation else z
    if version == "B":
        y = (linear0(x, w0, b0) + y).astype(np.float32)
    return quantize(y, out_mode), z, k


def embeddings_linear_forward(x, edges, inv_w, n_bins, W, W1, b1=None, *, version="A", activation=False,
                              bias=None, w0=None, b0=None, mode="bf16", out_mode="f32"):
    """The module output fed to ``flatten`` + ``nn.Linear(F * D, H)`` under bf16
    autocast (the consumer step after ``module.py:207-248``; the reference has no
    fused counterpart).

    The Linear sees the module output rounded to bf16 (``mode`` "bf16": the
    autocast module output; "f32": the fp32 output, rounded for the product) and
    its weight rounded to bf16; the product is accumulated exactly here (float64)
    and rounded to ``out_mode``.  Returns ``(z, e, scale)``: the output ``[N, H]``,
    the bf16 embeddings ``[N, F, D]`` and ``|e| @ |W1|^T`` (the magnitude that
    bounds the rounding error of each output, for tolerances).
    """
    e, _, _ = embeddings_forward(x, edges, inv_w, n_bins, W, version=version, activation=activation,
                                 bias=bias, w0=w0, b0=b0, mode=mode, out_mode="bf16")
    n = e.shape[0]
    e2 = e.reshape(n, -1).astype(np.float64)
    w = bf16_round(np.asarray(W1, np.float32)).astype(np.float64)
    z = e2 @ w.T
    if b1 is not None:
        z = z + np.asarray(b1, np.float64)[None]
    with np.errstate(invalid="ignore"):
        scale = np.abs(e2) @ np.abs(w).T
    return quantize(z.astype(np.float32), out_mode), e, scale


def embeddings_backward(g, x, edges, inv_w, n_bins, W, *, version="A", activation=False,
                        bias=None, w0=None, b0=None, mode="f32"):
    """Autograd of ``embeddings_forward``.

    ReLU blocks the gradient where its input is ``<= 0`` and passes it
    elsewhere, NaN inputs included (torch ``threshold_backward``). The x_ple branch receives ``q(g * mask)``: under
    autocast the gradient of the low-precision ``x_ple`` is cast to that type
    before the reference backward op (``_autograd.py:68-80``). The bias and
    linear0 gradients are fp32 reductions of the unrounded gradient.
    Returns a dict with ``grad_x``, ``grad_W`` and ``grad_bias`` (A) or
    ``grad_w0``/``grad_b0`` (B), all float64.
    """
    g = np.asarray(g, dtype=np.float32)
    x = np.asarray(x, dtype=np.float32)
    _, z, _ = embeddings_forward(x, edges, inv_w, n_bins, W, version=version,
                                 activation=activation, bias=bias, w0=w0, b0=b0,
                                 mode=mode)
    g_ple = np.where(z <= 0, np.float32(0.0), g) if activation else g
    g_ple = g_ple.astype(np.float32)
    grad_x, grad_W, abs_W = x_ple_backward(quantize(g_ple, mode), x, edges, inv_w, n_bins, W, mode,
                                           with_abs=True)
    out = {"grad_W": grad_W, "abs": {"grad_W": abs_W}}
    g64 = g.astype(np.float64)
    if version == "A":
        out["grad_bias"] = g_ple.astype(np.float64).sum(axis=0)
        out["abs"]["grad_bias"] = np.abs(g_ple.astype(np.float64)).sum(axis=0)
    else:
        x64 = x.astype(np.float64)
        out["grad_w0"] = np.einsum("nfd,nf->fd", g64, x64)
        out["grad_b0"] = g64.sum(axis=0)
        out["abs"]["grad_w0"] = np.einsum("nfd,nf->fd", np.abs(g64), np.abs(x64))
        out["abs"]["grad_b0"] = np.abs(g64).sum(axis=0)
        grad_x = grad_x + np.einsum("nfd,fd->nf", g64, w0.astype(np.float64))
    out["grad_x"] = grad_x
    return out


# fp32 summation allowance: any fp32 summation order of n terms differs from the
# exact sum by up to ~n*u*sum|terms| (u = 2**-24); batch reductions are compared
# with 2**-20 * sum|terms| added to the element tolerance.
SUM_ALLOWANCE = 2.0 ** -20


def assert_reduction_close(got, ref, abs_sum, rtol=1e-4, atol=1e-5, err_msg=""):
    """Element-wise ``|got - ref| <= atol + rtol*|ref| + SUM_ALLOWANCE*sum|terms|``."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    bound = atol + rtol * np.abs(ref) + SUM_ALLOWANCE * np.asarray(abs_sum, np.float64)
    bad = ~(np.abs(got - ref) <= bound)
    if bad.any():
        idx = np.argwhere(bad)[:5].tolist()
        raise AssertionError(
            f"{err_msg}: {int(bad.sum())} of {bad.size} elements outside the tolerance; first {idx}: "
            f"got {got[bad][:5]}, ref {ref[bad][:5]}, bound {bound[bad][:5]}"
        )


# ---------------------------------------------------------------------------
# Dense formulation of the upstream algorithm (independent cross-check)
# ---------------------------------------------------------------------------

def dense_encoding(x, edges, inv_w, n_bins):
    """Clamped piecewise-linear encoding ``[N, F, B]`` in the physical layout.

    Column ``j < n-1`` holds logical bin ``j``; column ``B-1`` holds the last
    real bin; the columns in between are masked to zero. Every column is
    ``(x - e_j) * r_j`` clamped to ``<= 1`` (first bin), ``[0, 1]`` (middle
    bins) or ``>= 0`` (last bin); a single-bin feature is unclamped
    (upstream ``PiecewiseLinearEncoding``; module.py:16-24).
    """
    x = np.asarray(x, dtype=np.float64)
    n, f = x.shape
    b_max = edges.shape[1] - 1
    enc = np.zeros((n, f, b_max))
    for i in range(f):
        nb = int(n_bins[i])
        for j in range(nb):
            col = b_max - 1 if j == nb - 1 else j
            v = (x[:, i] - edges[i, j]) * inv_w[i, j]
            if nb > 1:
                if j == 0:
                    v = np.minimum(v, 1.0)
                elif j == nb - 1:
                    v = np.maximum(v, 0.0)
                else:
                    v = np.clip(v, 0.0, 1.0)
            enc[:, i, col] = v
    return enc


def dense_forward(x, edges, inv_w, n_bins, W, *, version="A", activation=False,
                  bias=None, w0=None, b0=None):
    """Upstream dense forward in float64: encoding, per-feature matmul, epilogue."""
    enc = dense_encoding(x, edges, inv_w, n_bins)
    y = np.einsum("nfb,fbd->nfd", enc, W.astype(np.float64))
    if version == "A" and bias is not None:
        y = y + bias[None]
    if activation:
        y = np.maximum(y, 0.0)
    if version == "B":
        y = y + np.asarray(x, np.float64)[..., None] * w0[None] + b0[None]
    return y


# ---------------------------------------------------------------- standalone encoding

def _encoding_bounds(j, nb):
    """Clamp bounds of logical column j of an nb-bin feature (upstream
    ``PiecewiseLinearEncoding``'s column clamps; the position formula is the
    reference's, backward_cuda.cu:194-196)."""
    if nb == 1:
        return -np.inf, np.inf
    if j == 0:
        return -np.inf, 1.0
    if j == nb - 1:
        return 0.0, np.inf
    return 0.0, 1.0


def encoding(x, edges, inv_w, n_bins, *, padded=False, dtype=np.float32):
    """Materialised encoding: ``[N, sum n_i]`` (feature-major, logical bin
    order) or, with ``padded``, ``[N, F, B]`` in the weights' physical layout.
    ``dtype=np.float32`` evaluates ``(x - e_j) * r_j`` in fp32 (the kernel's
    arithmetic); ``np.float64`` in double precision.  NaN propagates through
    the clamps."""
    x = np.asarray(x, dtype=dtype)
    n, f = x.shape
    b_max = edges.shape[1] - 1
    cols = []
    out = np.zeros((n, f, b_max), dtype=dtype) if padded else None
    for i in range(f):
        nb = int(n_bins[i])
        for j in range(nb):
            v = (x[:, i] - dtype(edges[i, j])) * dtype(inv_w[i, j])
            lo, hi = _encoding_bounds(j, nb)
            v = np.where(v < lo, dtype(lo), v)
            v = np.where(v > hi, dtype(hi), v)
            if padded:
                out[:, i, b_max - 1 if j == nb - 1 else j] = v
            else:
                cols.append(v)
    return out if padded else np.stack(cols, axis=1).astype(dtype)


def encoding_grad_x(g, x, edges, inv_w, n_bins, *, padded=False):
    """``grad_x[b, i] = sum_j g[b, col(i, j)] * r_j * [lo_j <= t_j <= hi_j]``
    with t_j in fp32 (the kernel's mask) and the sum in float64; returns
    ``(grad_x, sum of |terms|)``."""
    x32 = np.asarray(x, dtype=np.float32)
    n, f = x32.shape
    b_max = edges.shape[1] - 1
    g = np.asarray(g, dtype=np.float64)
    gx = np.zeros((n, f))
    ab = np.zeros((n, f))
    c = 0
    for i in range(f):
        nb = int(n_bins[i])
        for j in range(nb):
            r = np.float32(inv_w[i, j])
            t = (x32[:, i] - np.float32(edges[i, j])) * r
            lo, hi = _encoding_bounds(j, nb)
            m = (t >= lo) & (t <= hi)
            col = g[:, i, b_max - 1 if j == nb - 1 else j] if padded else g[:, c + j]
            term = np.where(m, col * np.float64(r), 0.0)
            gx[:, i] += term
            ab[:, i] += np.abs(term)
        c += nb
    return gx, ab


# ---------------------------------------------------------------- bin edges

def quantile_bins(X, n_bins):
    """Quantile bin edges per feature (upstream ``compute_bins`` without a
    tree): ``unique(quantile(X[:, i], linspace(0, 1, n_bins + 1)))`` with
    linear interpolation, in float64."""
    X = np.asarray(X, dtype=np.float64)
    qs = np.linspace(0.0, 1.0, n_bins + 1)
    return [np.unique(np.quantile(X[:, i], qs, method="linear")) for i in range(X.shape[1])]
