"""Host-side logic of bench.py, on CPU: the committed ncu DRAM-traffic captures
it reads for the roofline line (parsing, scaling to a launch's rows, and their
ratio to the algorithmic bytes), and the reference arm's JSON line."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def test_traffic_lines_parse_and_scale_with_rows():
    import bench

    for cfg in ("c5", "c4"):
        for kernel in ("forward", "backward"):
            one = bench.read_traffic(cfg, kernel, 1000)
            assert one is not None and one > 0, (cfg, kernel)
            assert bench.read_traffic(cfg, kernel, 3000) == pytest.approx(3 * one)
    assert bench.read_traffic("c5", "no-such-kernel", 10) is None


@pytest.mark.parametrize("cfg", ["c5", "c4"])
def test_captured_traffic_is_close_to_the_algorithmic_bytes(cfg):
    """The committed captures of the shipped kernels move at most 1.1x the bytes a launch must move
    (re-reads would show above it); the forward's captures may fall a little short, the end of its
    output still being in L2 when the captured launch ends."""
    import bench
    from piecewiselinearembeddings_optimized_b200 import workloads

    n = 65536
    wl = workloads.make_workload(cfg, n=8)
    alg = workloads.algorithmic_bytes(wl, n_local=n)
    bwd = bench.read_traffic(cfg, "backward", n)
    fwd = bench.read_traffic(cfg, "forward", n)
    assert 0.95 * alg["bwd"] <= bwd <= 1.1 * alg["bwd"], (bwd, alg["bwd"])
    assert 0.85 * alg["fwd"] <= fwd <= 1.1 * alg["fwd"], (fwd, alg["fwd"])


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run(
        [sys.executable, "bench.py", "--impl", "reference", "--config", "c1", "--steps", "1", "--warmup", "1",
         "--no-reference-cuda"],
        cwd=ROOT, capture_output=True, text=True, timeout=600,
    )
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["unit"] == "feature-embeddings/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 1
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"] == "c1"
