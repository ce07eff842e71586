"""Timed CPU baseline for the PLE path (TEST / MEASUREMENT INFRASTRUCTURE ONLY).

The reference's CPU path is its base class from ``rtdl_num_embeddings==0.0.12``
(``module.py:222-223`` delegates non-CUDA inputs to ``super().forward``),
which is not installed here.  This module restates that upstream dense
algorithm with torch CPU ops - clamped ``[n, F, B]`` encoding, per-feature
contraction with ``weight[F, B, D]``, bias / ReLU / ``linear0`` epilogue and
autograd for the backward - and times one forward+backward step on a
bounded sample of a workload's rows with every host thread torch may use.
Used only by ``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference``).
"""
from __future__ import annotations

import os
import time

import numpy as np
import torch


def _encoding(x, left, inv_w, lo, hi, col):
    """Clamped encoding in the physical layout (see ``ple_oracle.dense_encoding``)."""
    t = (x[:, :, None] - left[None]) * inv_w[None]
    return torch.maximum(torch.minimum(t, hi[None]), lo[None]) * col[None]


def _tables(bins, max_n_bins):
    """Per physical column: left edge, inverse width, clamp bounds and mask.

    First bin ``(-inf, 1]``, middle bins ``[0, 1]``, last bin ``[0, inf)``, a
    single-bin feature unclamped, padding columns masked to zero."""
    f = len(bins)
    left = np.zeros((f, max_n_bins), np.float32)
    inv = np.zeros((f, max_n_bins), np.float32)
    lo = np.zeros((f, max_n_bins), np.float32)
    hi = np.zeros((f, max_n_bins), np.float32)
    col = np.zeros((f, max_n_bins), np.float32)
    for i, e in enumerate(bins):
        e = np.asarray(e, np.float32)
        n = e.size - 1
        r = (np.float32(1.0) / (e[1:] - e[:-1])).astype(np.float32)
        for j in range(n):
            c = max_n_bins - 1 if j == n - 1 else j
            left[i, c], inv[i, c], col[i, c] = e[j], r[j], 1.0
            lo[i, c] = -np.inf if (j == 0 or n == 1) else 0.0
            hi[i, c] = np.inf if (j == n - 1) else 1.0
    return tuple(torch.from_numpy(a) for a in (left, inv, lo, hi, col))


def dense_step(x, tables, weight, bias, w0, b0, activation, g):
    """One upstream-style forward + backward on CPU; returns the output."""
    enc = _encoding(x, *tables)
    y = torch.einsum("nfb,fbd->nfd", enc, weight)
    if bias is not None:
        y = y + bias
    if activation:
        y = torch.relu(y)
    if w0 is not None:
        y = torch.addcmul(b0, w0, x[..., None]) + y
    y.backward(g)
    return y


def time_cpu_baseline(wl, n_sample: int, steps: int = 3, warmup: int = 1, threads: int | None = None) -> dict:
    """Time ``steps`` dense fp32 fwd+bwd steps on ``n_sample`` rows of ``wl``.

    Returns feature-embeddings/s (``n_sample * F / seconds_per_step``), the
    threads used and a description of the sample.
    """
    threads = threads or len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    n_sample = min(n_sample, wl.n)
    b = wl.max_n_bins
    tables = _tables(wl.bins, b)
    x = torch.from_numpy(np.ascontiguousarray(wl.x[:n_sample])).requires_grad_(True)
    weight = torch.from_numpy(wl.weight).requires_grad_(True)
    bias = None if wl.bias is None else torch.from_numpy(wl.bias).requires_grad_(True)
    w0 = None if wl.w0 is None else torch.from_numpy(wl.w0).requires_grad_(True)
    b0 = None if wl.b0 is None else torch.from_numpy(wl.b0).requires_grad_(True)
    gen = torch.Generator().manual_seed(7)
    g = torch.randn((n_sample, wl.f, wl.d), generator=gen)
    for _ in range(warmup):
        dense_step(x, tables, weight, bias, w0, b0, wl.activation, g)
    times = []
    for _ in range(steps):
        for p in (x, weight, bias, w0, b0):
            if p is not None:
                p.grad = None
        t0 = time.perf_counter()
        dense_step(x, tables, weight, bias, w0, b0, wl.activation, g)
        times.append(time.perf_counter() - t0)
    sec = float(np.median(times))
    return {
        "value": n_sample * wl.f / sec,
        "unit": "feature-embeddings/s",
        "cores": threads,
        "seconds_per_step": sec,
        "sample": f"{n_sample} of {wl.n} rows of {wl.name}, dense fp32 fwd+bwd (torch CPU, "
                  f"upstream algorithm restated), median of {steps} steps",
    }
