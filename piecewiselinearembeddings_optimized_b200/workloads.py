"""Seeded synthetic workloads for the five benchmark configurations.

No dataset is named for this path; every input is synthetic with the shapes,
distributions and seeds of the benchmark configurations:

* ``c1`` 1024 x 8 features, 16 bins, D=16, fp32, version B + ReLU;
* ``c2`` 4096 x 64, 48 bins, D=32, fp32, version A, no activation, mixed
  N(0,1) / LogNormal(0,1) / U(-5,5) features;
* ``c3`` 16384 x 128, ragged 2..64 bins, D=64, fp32, version B + ReLU, a
  quarter of the features integer-valued Poisson(3) with collapsed edges;
* ``c4`` 65536 x 256, 32 bins, D=24, bf16 output / fp32 accumulation,
  version B + ReLU, 1% of x set to +-10, bf16 upstream gradient;
* ``c5`` 1,048,576 (global, sharded over ranks) x 512, 64 bins, D=16, fp32,
  version B + ReLU.

Edges are evenly spaced quantiles of a seeded draw of each feature's law.
Parameters follow the reference benchmark's initialisation
(``tests/test_ple_cuda_benchmark.py:357-387``): ``W ~ U(0.05, 0.25)``,
``bias ~ U(0.05, 0.20)``, ``w0 ~ U(-0.2, 0.2)``, ``b0 ~ U(-0.1, 0.1)``.
Everything is numpy and float32 so the same bytes are produced on any host.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

CONFIG_NAMES = ("c1", "c2", "c3", "c4", "c5")


@dataclass
class Workload:
    name: str
    n: int
    f: int
    d: int
    version: str
    activation: bool
    mode: str          # arithmetic mode of x_ple: "f32" or "bf16"
    out_mode: str      # storage type of the output and of the upstream gradient
    bins: list = field(repr=False)
    x: np.ndarray = field(repr=False)
    weight: np.ndarray = field(repr=False)
    bias: np.ndarray | None = field(repr=False, default=None)
    w0: np.ndarray | None = field(repr=False, default=None)
    b0: np.ndarray | None = field(repr=False, default=None)
    seed: int = 0

    @property
    def max_n_bins(self) -> int:
        return max(len(b) - 1 for b in self.bins)

    def describe(self) -> dict:
        return {
            "workload": self.name, "batch": self.n, "n_features": self.f,
            "max_n_bins": self.max_n_bins, "d_embedding": self.d, "version": self.version,
            "activation": self.activation, "x_ple_mode": self.mode, "out_dtype": self.out_mode,
        }


def _quantile_edges(draw: np.ndarray, n_bins: int, dedup: bool) -> np.ndarray:
    q = np.quantile(draw.astype(np.float64), np.linspace(0.0, 1.0, n_bins + 1))
    q = q.astype(np.float32)
    if dedup:
        q = np.unique(q)
        if q.size < 2:
            q = np.array([q[0], q[0] + 1.0], dtype=np.float32)
    return q


def _params(f, b, d, version, seed=42):
    rng = np.random.default_rng(seed)
    w = rng.uniform(0.05, 0.25, size=(f, b, d)).astype(np.float32)
    if version == "A":
        bias = rng.uniform(0.05, 0.20, size=(f, d)).astype(np.float32)
        return w, bias, None, None
    w0 = rng.uniform(-0.2, 0.2, size=(f, d)).astype(np.float32)
    b0 = rng.uniform(-0.1, 0.1, size=(f, d)).astype(np.float32)
    return w, None, w0, b0


def make_bins(name: str, seed: int = 1234, f: int | None = None) -> list[np.ndarray]:
    """Edges of a configuration (independent of batch size)."""
    rng = np.random.default_rng(seed)
    if name == "c1":
        return [_quantile_edges(rng.standard_normal(10_000), 16, False) for _ in range(f or 8)]
    if name == "c2":
        out = []
        for i in range(f or 64):
            out.append(_quantile_edges(_draw_c2(rng, i, 50_000), 48, False))
        return out
    if name == "c3":
        f = f or 128
        counts = rng.integers(2, 65, size=f)
        counts[1] = 64                       # one N(0,1) feature pins max_n_bins = 64
        out = []
        for i in range(f):
            if i % 4 == 0:                   # a quarter: integer-valued Poisson(3)
                draw = rng.poisson(3.0, size=100_000).astype(np.float32)
                out.append(_quantile_edges(draw, int(counts[i]), True))
            else:
                out.append(_quantile_edges(rng.standard_normal(100_000), int(counts[i]), False))
        return out
    if name == "c4":
        return [_quantile_edges(rng.standard_normal(100_000), 32, False) for _ in range(f or 256)]
    if name == "c5":
        return [_quantile_edges(rng.standard_normal(200_000), 64, False) for _ in range(f or 512)]
    raise ValueError(name)


def _draw_c2(rng, i, size):
    if i % 3 == 0:
        return rng.standard_normal(size)
    if i % 3 == 1:
        return rng.lognormal(0.0, 1.0, size)
    return rng.uniform(-5.0, 5.0, size)


SPECS = {
    #       n          f    d   version relu   mode    out
    "c1": (1024,       8,   16, "B", True,  "f32",  "f32"),
    "c2": (4096,       64,  32, "A", False, "f32",  "f32"),
    "c3": (16384,      128, 64, "B", True,  "f32",  "f32"),
    "c4": (65536,      256, 24, "B", True,  "bf16", "bf16"),
    "c5": (1_048_576,  512, 16, "B", True,  "f32",  "f32"),
}


def make_x(name: str, n: int, f: int, seed: int, rank: int = 0) -> np.ndarray:
    """Input batch ``[n, f]`` float32 (rank selects a disjoint seeded shard)."""
    rng = np.random.default_rng([seed, rank])
    if name == "c2":
        x = np.empty((n, f), dtype=np.float32)
        for i in range(f):
            x[:, i] = _draw_c2(rng, i, n)
        return x
    if name == "c3":
        x = rng.standard_normal((n, f), dtype=np.float32)
        for i in range(0, f, 4):
            x[:, i] = rng.poisson(3.0, size=n).astype(np.float32)
        return x
    x = rng.standard_normal((n, f), dtype=np.float32)
    if name == "c4":
        m = rng.random((n, f)) < 0.01
        x[m] = np.where(rng.random(int(m.sum())) < 0.5, -10.0, 10.0).astype(np.float32)
    return x


def make_workload(name: str, n: int | None = None, f: int | None = None, rank: int = 0,
                  seed: int = 0) -> Workload:
    """Build a configuration; ``n``/``f`` override the batch / feature count."""
    n0, f0, d, version, relu, mode, out_mode = SPECS[name]
    n = n0 if n is None else n
    f = f0 if f is None else f
    bins = make_bins(name, f=f)
    b = max(len(e) - 1 for e in bins)
    w, bias, w0, b0 = _params(f, b, d, version)
    x = make_x(name, n, f, seed, rank)
    return Workload(name, n, f, d, version, relu, mode, out_mode, bins, x, w, bias, w0, b0, seed)


def make_grad(wl: Workload, seed: int = 7, rank: int = 0) -> np.ndarray:
    """Upstream gradient ``g ~ N(0, 1)`` of shape ``[n, f, d]`` (float32 values;
    rounded to bf16 when the configuration's output is bf16)."""
    rng = np.random.default_rng([seed, rank])
    g = rng.standard_normal((wl.n, wl.f, wl.d), dtype=np.float32)
    if wl.out_mode == "bf16":
        bits = g.view(np.uint32).astype(np.uint64)
        g = (((bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)).view(np.float32)
    return g


def algorithmic_bytes(wl: Workload, n_local: int | None = None) -> dict:
    """HBM bytes one fused forward+backward step must move at minimum.

    fwd = x + edges + W + epilogue params + output;
    bwd = g + x + edges + W (read) + epilogue params + grad_x + grad_W + param grads.
    Bin indices, workspaces and re-reads are not counted.
    """
    n = wl.n if n_local is None else n_local
    f, b, d = wl.f, wl.max_n_bins, wl.d
    s_out = 2 if wl.out_mode in ("bf16", "f16") else 4
    p = 4 * f * d if wl.version == "A" else 8 * f * d
    edges = 4 * f * (b + 1)
    w = 4 * f * b * d
    fwd = 4 * n * f + edges + w + p + n * f * d * s_out
    bwd = n * f * d * s_out + 4 * n * f + edges + w + p + 4 * n * f + w + p
    return {"fwd": fwd, "bwd": bwd, "step": fwd + bwd}
