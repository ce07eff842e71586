"""Benchmark: fused PLE forward+backward, feature-embeddings/s and HBM GB/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c5|c4|...] [--impl ours|reference]

One step = the fused forward kernel, the fused backward (kernel + finalize)
and, with N > 1, one NCCL all-reduce of the packed parameter gradients.
Under torchrun each rank processes its shard of the configuration's global
batch (c5: 1,048,576 rows split evenly).  Timing: W warm-up steps, then K
steps between barrier + synchronize, CUDA events on the compute stream, max
over ranks.  Inputs (x, upstream gradient) are resident in HBM for ``value``;
``e2e`` repeats the step through the drop-in module with x copied from
pinned host memory and the gradients read back every step; the copy of the
next step's x runs on a second stream while the current step computes
(double-buffered device x), all copies inside the timed region.  Every step
moves far more than the 126 MB L2 (c5: ~9 GB per GPU at N=8), so no L2 flush
is inserted.  ``--impl reference`` times the CPU stand-in for the
reference's CPU path (upstream dense algorithm, torch CPU, all host
threads) on a bounded row sample and prints the same metric.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "PLE fwd+bwd feature-embeddings/sec & HBM GB/s vs ~8 TB/s at 1/2/4/8 B200"
UNIT = "feature-embeddings/s"
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c5")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=None, help="override the global batch (profiling runs)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-c4", action="store_true", help="skip the c4 north-star figures of the default run")
    ap.add_argument("--no-reference-cuda", action="store_true",
                    help="reference arm: skip the GPU timing of the reference's own CUDA ops")
    ap.add_argument("--consumer", type=int, default=None, metavar="H",
                    help="time the module fused into a following Linear(F*D -> H) (forward, bf16 autocast "
                         "semantics) against the unfused embeddings kernel + cuBLAS, one GPU")
    return ap.parse_args()


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return FALLBACK_HBM_GBS, "fallback"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        # wait for nvidia-smi's first sample so that the timed region is covered from its start
        self.n_pre = 0
        deadline = time.time() + 5.0
        while self.proc is not None and time.time() < deadline:
            lines = Path(self.path).read_text().splitlines()
            if lines:
                self.n_pre = len(lines)
                break
            time.sleep(0.01)
        self.t0 = time.time()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        # samples taken after the timed region began; the last pre-start sample if the region was shorter
        # than the sampling period
        rows = rows[self.n_pre:] or rows[-1:]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[j] for r in rows for j in range(4) if r[5 + j].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def gpu_id(torch, dev, local):
    """nvidia-smi id of this rank's GPU (its UUID, robust to CUDA_VISIBLE_DEVICES)."""
    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:  # noqa: BLE001
        return str(local)


def reference_arm(args, ws, rank):
    """CPU stand-in for the reference's CPU path (rank 0 only)."""
    if rank != 0:
        return 0
    from oracle.cpu_baseline import time_cpu_baseline
    from piecewiselinearembeddings_optimized_b200 import workloads

    n_global = workloads.SPECS[args.config][0]
    sample = {"c1": 1024, "c2": 2048, "c3": 512, "c4": 1024, "c5": 1024}[args.config]
    wl = workloads.make_workload(args.config, n=sample)
    t0 = time.time()
    res = time_cpu_baseline(wl, sample, steps=max(1, args.steps), warmup=max(1, args.warmup))
    line = {
        "impl": "reference", "metric": METRIC, "value": res["value"], "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["seconds_per_step"] * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": config_block(args.config, n_global, args.gpus),
        "cpu_baseline": {"value": res["value"], "unit": UNIT, "cores": res["cores"], "kind": "port",
                         "sample": res["sample"]},
        "e2e": {"value": res["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference CPU path = upstream rtdl_num_embeddings (not installable offline); timed here as "
                "its dense algorithm restated in torch CPU ops (oracle/cpu_baseline.py)",
    }
    if not args.no_reference_cuda:
        line["reference_cuda"] = reference_cuda_timings(args)
    line["wall_s"] = round(time.time() - t0, 1)
    print(json.dumps(line), flush=True)
    return 0


def reference_cuda_timings(args) -> dict:
    """The reference's own CUDA ops (compiled from its sources into oracle/_ref) timed on GPU 0 for the
    c4 shape and the per-GPU shard of c5 at 8 GPUs (131,072 rows; the reference's unfused epilogue
    holds several [N, F, D] temporaries, too many for the full 1,048,576-row batch), each in its own
    process (the reference registers the same op namespace as this project).  A secondary, GPU-side
    baseline reported beside the CPU figure; `value` stays the CPU figure."""
    out = {}
    script = ROOT / "oracle" / "time_reference_cuda.py"
    for key, cfg, batch in (("c4", "c4", None), ("c5_shard_of_8", "c5", 131072)):
        cmd = [sys.executable, str(script), "--config", cfg, "--steps", str(max(5, args.steps)),
               "--warmup", str(max(3, args.warmup))]
        if batch:
            cmd += ["--batch", str(batch)]
        try:
            r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
            lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
            out[key] = json.loads(lines[-1]) if (r.returncode == 0 and lines) else {
                "unavailable": f"exit {r.returncode}: {(r.stderr or r.stdout).strip()[-300:]}"}
        except (OSError, subprocess.TimeoutExpired, ValueError) as e:
            out[key] = {"unavailable": f"{type(e).__name__}: {e}"}
    return out


def consumer_bench(args) -> int:
    """The embeddings fused into the consumer's first Linear(F * D -> H): one step = one forward
    (rtdl_num_embeddings_cuda::embeddings_linear_forward through the C ABI, bf16 autocast semantics,
    bf16 output) over the configuration's batch; the same step unfused (the module's own fused kernel
    writing [N, F, D] bf16, then cuBLAS addmm) is timed beside it.  Roofline: tensor (2 N F D H flop
    per launch against the measured bf16 GEMM peak)."""
    import torch

    import rtdl_num_embeddings_cuda  # noqa: F401
    from piecewiselinearembeddings_optimized_b200 import _native, workloads
    from piecewiselinearembeddings_optimized_b200.module import pad_bin_tables

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    name, H = args.config, int(args.consumer)
    n0, F, D, version, relu, _mode, _out = workloads.SPECS[name]
    N = args.batch or min(n0, 131072)
    wl = workloads.make_workload(name, n=8)
    B = wl.max_n_bins
    edges, inv_w, n_bins = [t.to(dev) for t in pad_bin_tables([torch.from_numpy(b) for b in wl.bins])]
    W = torch.from_numpy(wl.weight).to(dev)
    t = lambda a: None if a is None else torch.from_numpy(a).to(dev)  # noqa: E731
    bias, w0, b0 = t(wl.bias), t(wl.w0), t(wl.b0)
    epi = 2 if version == "B" else 1
    gen = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(N, F, device=dev, generator=gen)
    w1 = (torch.randn(H, F * D, device=dev, generator=gen) / (F * D) ** 0.5).to(torch.bfloat16)
    b1 = torch.randn(H, device=dev, generator=gen) * 0.1
    z = torch.empty(N, H, device=dev, dtype=torch.bfloat16)
    lib = _native.capi()
    ws_bytes = lib.ple_embeddings_linear_workspace_size(F, B, D, H, _native.DTYPE_BF16)
    if ws_bytes == 0:
        print(json.dumps({"error": "unsupported consumer shape"}))
        return 1
    wsp = torch.empty(ws_bytes + 256, dtype=torch.uint8, device=dev)
    wsa = (wsp.data_ptr() + 255) // 256 * 256
    sp = torch.cuda.current_stream(dev).cuda_stream
    P = lambda a: None if a is None else a.data_ptr()  # noqa: E731
    ops = torch.ops.rtdl_num_embeddings_cuda
    b1h = b1.to(torch.bfloat16)

    def fused():
        _native.check(lib.ple_embeddings_linear_forward(
            x.data_ptr(), edges.data_ptr(), inv_w.data_ptr(), n_bins.data_ptr(), W.data_ptr(), P(bias), P(w0),
            P(b0), epi, int(relu), _native.DTYPE_BF16, N, F, B, D, w1.data_ptr(), _native.DTYPE_BF16,
            b1.data_ptr(), H, _native.DTYPE_BF16, z.data_ptr(), wsa, ws_bytes, sp), "embeddings_linear_forward")

    def unfused():
        e = ops.embeddings_forward(x, edges, inv_w, n_bins, W, bias, w0, b0, epi, relu, torch.bfloat16,
                                   torch.bfloat16)
        torch.addmm(b1h, e.view(N, -1), w1.t(), out=z)

    def timed(fn):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize(dev)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for a, b in ev:
            a.record()
            fn()
            b.record()
        torch.cuda.synchronize(dev)
        return float(np.median([a.elapsed_time(b) for a, b in ev]))

    clocks = ClockSampler(gpu_id(torch, dev, 0))
    clocks.start()
    time.sleep(0.05)
    t_fused = timed(fused)
    t_unfused = timed(unfused)
    clock_info = clocks.stop()
    status = lib.ple_linear_status()
    flop = 2.0 * N * F * D * H
    peak = None
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        peak = float(json.loads(p.read_text()).get("bf16_tflops", 0)) or None
    achieved = flop / (t_fused * 1e-3) / 1e12
    line = {
        "metric": f"PLE + Linear(F*D -> {H}) forward feature-embeddings/s (fused consumer)",
        "value": N * F / (t_fused * 1e-3), "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t_fused, "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{name} shapes (N={N}, F={F}, B={B}, D={D}) -> Linear({F * D}, {H})",
                   "inputs": "x [N, F] fp32 and the bf16 linear weight resident in HBM"},
        "unfused_ms_per_step": t_unfused, "speedup_vs_unfused": t_unfused / t_fused,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": (achieved / peak) if peak else None, "peak_source": "measured" if peak else None},
        "status_word": status, "clocks": clock_info,
    }
    print(json.dumps(line))
    return 0 if status == 0 else 1


def north_star_c4(torch, dev, lib, steps, warmup, peak):
    """The north-star target shape timed beside the headline workload (one GPU): configuration c4
    (65,536 x 256, 32 bins, D = 24, bf16 output and upstream gradient, version B + ReLU), one step =
    the fused forward then the fused backward (kernel + finalize) with every input resident in HBM,
    CUDA events on the compute stream.  Target: >= 70 % of the HBM roofline, i.e. a step of at most
    324 us at 8 TB/s, 401 us at the measured copy bandwidth."""
    from piecewiselinearembeddings_optimized_b200 import _native, workloads
    from piecewiselinearembeddings_optimized_b200.module import pad_bin_tables

    n0, F, D, version, relu, mode, out_mode = workloads.SPECS["c4"]
    wl = workloads.make_workload("c4", n=8)
    B = wl.max_n_bins
    edges, inv_w, n_bins = [t.to(dev) for t in pad_bin_tables([torch.from_numpy(b) for b in wl.bins])]
    W = torch.from_numpy(wl.weight).to(dev)
    w0, b0 = torch.from_numpy(wl.w0).to(dev), torch.from_numpy(wl.b0).to(dev)
    gen = torch.Generator(device=dev).manual_seed(4000)
    x = torch.randn(n0, F, device=dev, generator=gen)
    m = torch.rand(n0, F, device=dev, generator=gen) < 0.01
    x[m] = torch.where(torch.rand(n0, F, device=dev, generator=gen) < 0.5, -10.0, 10.0)[m]
    g = torch.randn(n0, F, D, device=dev, generator=gen).to(torch.bfloat16)
    y = torch.empty(n0, F, D, device=dev, dtype=torch.bfloat16)
    gx = torch.empty(n0, F, device=dev)
    gW = torch.empty(F, B, D, device=dev)
    gw0, gb0 = torch.empty(F, D, device=dev), torch.empty(F, D, device=dev)
    ws_bytes = lib.ple_backward_workspace_size(n0, F, B, D)
    wsp = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    sp = torch.cuda.current_stream(dev).cuda_stream
    bf = _native.DTYPE_BF16

    def fwd():
        _native.check(lib.ple_embeddings_forward(
            x.data_ptr(), edges.data_ptr(), inv_w.data_ptr(), n_bins.data_ptr(), W.data_ptr(), None, w0.data_ptr(),
            b0.data_ptr(), 2, 1, bf, n0, F, B, D, bf, y.data_ptr(), 3, None, sp), "c4 forward")

    def bwd():
        _native.check(lib.ple_embeddings_backward(
            g.data_ptr(), bf, x.data_ptr(), edges.data_ptr(), inv_w.data_ptr(), n_bins.data_ptr(), W.data_ptr(), None,
            w0.data_ptr(), b0.data_ptr(), 2, 1, bf, n0, F, B, D, None, 3, gx.data_ptr(), gW.data_ptr(), None,
            gw0.data_ptr(), gb0.data_ptr(), wsp.data_ptr(), ws_bytes, sp), "c4 backward")

    for _ in range(max(3, warmup)):
        fwd()
        bwd()
    torch.cuda.synchronize(dev)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    for k in range(steps):
        ev[k][0].record()
        fwd()
        ev[k][1].record()
        bwd()
        ev[k][2].record()
    torch.cuda.synchronize(dev)
    fwd_ms = float(np.median([e[0].elapsed_time(e[1]) for e in ev]))
    bwd_ms = float(np.median([e[1].elapsed_time(e[2]) for e in ev]))
    step_ms = float(np.median([e[0].elapsed_time(e[2]) for e in ev]))
    wb = workloads.algorithmic_bytes(wl, n_local=n0)
    step_gbs = wb["step"] / (step_ms * 1e-3) / 1e9
    return {
        "workload": "c4: 65536 x 256 features, 32 bins, D=24, bf16 output and gradient, version B + ReLU",
        "ms_per_step": step_ms, "us_per_step": step_ms * 1e3, "target_us_8tbs": wb["step"] / 8000e9 / 0.7 * 1e6,
        "target_us_measured_peak": wb["step"] / (peak * 1e9) / 0.7 * 1e6,
        "feature_embeddings_per_s": n0 * F / (step_ms * 1e-3), "step_gb_per_s": step_gbs,
        "step_frac_of_measured": step_gbs / peak, "step_frac_of_8tbs": step_gbs / 8000.0,
        "kernels": {"forward": {"ms": fwd_ms, "gb_per_s": wb["fwd"] / (fwd_ms * 1e-3) / 1e9,
                                "frac": wb["fwd"] / (fwd_ms * 1e-3) / 1e9 / peak},
                    "backward": {"ms": bwd_ms, "gb_per_s": wb["bwd"] / (bwd_ms * 1e-3) / 1e9,
                                 "frac": wb["bwd"] / (bwd_ms * 1e-3) / 1e9 / peak}},
        "timing": f"median of {steps} steps after {max(3, warmup)} warm-up steps, CUDA events; inputs resident in HBM",
    }


def config_block(name, n_global, ws):
    from piecewiselinearembeddings_optimized_b200 import workloads

    n0, f, d, version, relu, mode, out = workloads.SPECS[name]
    return {"workload": name, "global_batch": n_global, "n_features": f, "d_embedding": d,
            "max_n_bins": {"c1": 16, "c2": 48, "c3": 64, "c4": 32, "c5": 64}[name], "version": version,
            "activation": relu, "x_ple_dtype": mode, "out_dtype": out, "parallelism": f"dp{ws}",
            "l2": "no flush: every step streams > 126 MB (inputs larger than L2)"}


def main() -> int:
    args = parse()
    ws, rank, local = dist_env()
    if args.impl == "reference":
        return reference_arm(args, ws, rank)
    if args.consumer:
        return consumer_bench(args)

    import torch
    import torch.distributed as dist

    import rtdl_num_embeddings_cuda  # noqa: F401  (registers the ops)
    from piecewiselinearembeddings_optimized_b200 import _native, workloads
    from piecewiselinearembeddings_optimized_b200.module import CudaPiecewiseLinearEmbeddings, pad_bin_tables

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    name = args.config
    n0, F, D, version, relu, mode, out_mode = workloads.SPECS[name]
    n_global = args.batch or n0
    n_local = n_global // ws + (1 if rank < n_global % ws else 0)
    wl_small = workloads.make_workload(name, n=8)  # bins and parameters (independent of the batch)
    B = wl_small.max_n_bins
    dt = {"f32": torch.float32, "bf16": torch.bfloat16}
    q_dtype, o_dtype = dt[mode], dt[out_mode]
    bins = [torch.from_numpy(b) for b in wl_small.bins]
    edges, inv_w, n_bins = [t.to(dev) for t in pad_bin_tables(bins)]
    W = torch.from_numpy(wl_small.weight).to(dev)
    bias = None if wl_small.bias is None else torch.from_numpy(wl_small.bias).to(dev)
    w0 = None if wl_small.w0 is None else torch.from_numpy(wl_small.w0).to(dev)
    b0 = None if wl_small.b0 is None else torch.from_numpy(wl_small.b0).to(dev)
    epi = 2 if version == "B" else 1

    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    x = torch.randn(n_local, F, device=dev, generator=gen)
    if name == "c4":
        m = torch.rand(n_local, F, device=dev, generator=gen) < 0.01
        x[m] = torch.where(torch.rand(n_local, F, device=dev, generator=gen) < 0.5, -10.0, 10.0)[m]
    g = torch.randn(n_local, F, D, device=dev, generator=gen).to(o_dtype)
    y = torch.empty(n_local, F, D, device=dev, dtype=o_dtype)
    gx = torch.empty(n_local, F, device=dev)
    n_param = F * B * D + (F * D if version == "A" else 2 * F * D)
    flat = torch.zeros(n_param, device=dev)
    gW = flat[: F * B * D].view(F, B, D)
    gb = flat[F * B * D:].view(F, D) if version == "A" else None
    gw0 = flat[F * B * D: F * B * D + F * D].view(F, D) if version == "B" else None
    gb0 = flat[F * B * D + F * D:].view(F, D) if version == "B" else None
    lib = _native.capi()
    ws_bytes = lib.ple_backward_workspace_size(n_local, F, B, D)
    wsp = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    code = {torch.float32: 0, torch.bfloat16: 2}
    P = lambda t: None if t is None else t.data_ptr()  # noqa: E731

    def fwd():
        _native.check(lib.ple_embeddings_forward(
            x.data_ptr(), edges.data_ptr(), inv_w.data_ptr(), n_bins.data_ptr(), W.data_ptr(), P(bias), P(w0),
            P(b0), epi, int(relu), code[q_dtype], n_local, F, B, D, code[o_dtype], y.data_ptr(), 3, None,
            sp), "forward")

    def bwd():
        _native.check(lib.ple_embeddings_backward(
            g.data_ptr(), code[o_dtype], x.data_ptr(), edges.data_ptr(), inv_w.data_ptr(), n_bins.data_ptr(),
            W.data_ptr(), P(bias), P(w0), P(b0), epi, int(relu), code[q_dtype], n_local, F, B, D, None, 3,
            gx.data_ptr(),
            gW.data_ptr(), P(gb), P(gw0), P(gb0), wsp.data_ptr(), ws_bytes, sp), "backward")

    def allreduce():
        if ws > 1:
            dist.all_reduce(flat)

    # ---------------- warm-up and timed region (device-resident inputs)
    for _ in range(args.warmup):
        fwd(); bwd(); allreduce()
    torch.cuda.synchronize(dev)
    if ws > 1:
        dist.barrier()
    clocks = ClockSampler(gpu_id(torch, dev, local))
    clocks.start()
    time.sleep(0.05)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    torch.cuda.synchronize(dev)
    if ws > 1:
        dist.barrier()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for k in range(args.steps):
        ev[k][0].record(stream)
        fwd()
        ev[k][1].record(stream)
        bwd()
        ev[k][2].record(stream)
        allreduce()
        ev[k][3].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    if ws > 1:
        dist.barrier()
    clk = clocks.stop()
    total_ms = t_start.elapsed_time(t_end)
    fwd_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / args.steps
    bwd_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / args.steps
    ar_ms = sum(e[2].elapsed_time(e[3]) for e in ev) / args.steps
    t = torch.tensor([total_ms, fwd_ms, bwd_ms, ar_ms], device=dev)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, fwd_ms, bwd_ms, ar_ms = [float(v) for v in t.tolist()]
    ms_per_step = total_ms / args.steps
    value = n_global * F / (ms_per_step * 1e-3)

    # ---------------- end to end through the drop-in module (host buffers)
    e2e = None
    if not args.no_e2e:
        mod = CudaPiecewiseLinearEmbeddings(bins, D, activation=relu, version=version).to(dev)
        with torch.no_grad():
            mod.linear.weight.copy_(W)
            if bias is not None:
                mod.linear.bias.copy_(bias)
            if w0 is not None:
                mod.linear0.weight.copy_(w0)
                mod.linear0.bias.copy_(b0)
        mod.output_dtype = o_dtype
        x_host = x.cpu().pin_memory()
        params = list(mod.parameters())
        out_host = torch.empty(n_param, pin_memory=True)
        flat2 = torch.zeros(n_param, device=dev)

        # inputs double-buffered: the copy of step i + 1's x runs on a second stream while step i
        # computes; every step's copy is issued after the start event and waited for before its step
        copy_stream = torch.cuda.Stream(dev)
        xbufs = [torch.empty_like(x) for _ in range(2)]
        ready = [torch.cuda.Event() for _ in range(2)]
        free = [torch.cuda.Event() for _ in range(2)]

        def issue_copy(i, after=None):
            b = i % 2
            with torch.cuda.stream(copy_stream):
                if after is not None:
                    copy_stream.wait_event(after)
                copy_stream.wait_event(free[b])
                xbufs[b].copy_(x_host, non_blocking=True)
                ready[b].record(copy_stream)

        def e2e_step(i):
            b = i % 2
            stream.wait_event(ready[b])
            xd = xbufs[b]
            for p in params:
                p.grad = None
            with torch.autocast("cuda", dtype=q_dtype, enabled=q_dtype != torch.float32):
                out = mod(xd)
            out.backward(g)
            torch.cat([p.grad.reshape(-1) for p in params], out=flat2)
            if ws > 1:
                dist.all_reduce(flat2)
            out_host.copy_(flat2, non_blocking=True)
            free[b].record(stream)

        def e2e_run(n, start=None):
            for b in range(2):
                free[b].record(stream)
            issue_copy(0, start)
            for i in range(n):
                if i + 1 < n:
                    issue_copy(i + 1)
                e2e_step(i)

        e2e_run(max(1, args.warmup))
        torch.cuda.synchronize(dev)
        if ws > 1:
            dist.barrier()
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        e2e_run(args.steps, a0)
        a1.record(stream)
        torch.cuda.synchronize(dev)
        if ws > 1:
            dist.barrier()
        te = torch.tensor([a0.elapsed_time(a1)], device=dev)
        if ws > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = float(te.item()) / args.steps
        e2e = {"value": n_global * F / (e2e_ms * 1e-3), "unit": UNIT, "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": int(x_host.numel() * 4), "d2h_bytes_per_step": int(n_param * 4),
               "path": "rtdl_num_embeddings_cuda.CudaPiecewiseLinearEmbeddings forward+autograd backward, "
                       "x from pinned host memory (copy of the next step's x overlapped with the current "
                       "step, double-buffered), parameter gradients read back every step"}
        del mod, x_host

    if ws > 1:
        dist.destroy_process_group()
    if rank != 0:
        return 0

    # ---------------- roofline of the dominant kernel
    peak, peak_kind = measured_peak()
    wl_bytes = workloads.algorithmic_bytes(wl_small, n_local=n_local)
    kernels = {
        "forward": {"ms": fwd_ms, "bytes": wl_bytes["fwd"], "gbs": wl_bytes["fwd"] / (fwd_ms * 1e-3) / 1e9},
        "backward": {"ms": bwd_ms, "bytes": wl_bytes["bwd"], "gbs": wl_bytes["bwd"] / (bwd_ms * 1e-3) / 1e9},
    }
    dom = max(kernels, key=lambda k: kernels[k]["ms"])
    traffic = read_traffic(name, dom, n_local)
    roofline = {"bound": "hbm", "kernel": dom, "achieved": kernels[dom]["gbs"], "peak": peak, "unit": "GB/s",
                "frac": kernels[dom]["gbs"] / peak, "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                if peak_kind == "measured" else "fallback 6650 GB/s",
                "traffic": traffic}
    step_gbs = wl_bytes["step"] / (ms_per_step * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16" if mode == "bf16" else "f32", "data": "synthetic",
        "config": config_block(name, n_global, ws),
        "hbm_gbs_per_gpu": step_gbs, "hbm_frac_of_measured": step_gbs / peak, "hbm_frac_of_8tbs": step_gbs / 8000.0,
        "kernels": {k: {"ms": round(v["ms"], 4), "gb_per_s": round(v["gbs"], 1),
                        "frac": round(v["gbs"] / peak, 4)} for k, v in kernels.items()},
        "allreduce_ms": ar_ms, "roofline": roofline, "clocks": clk,
        "gpu_launches": 3 * args.steps, "e2e": e2e,
    }
    if ws == 1 and name == "c5" and not args.no_c4:
        line["north_star_c4"] = north_star_c4(torch, dev, lib, max(10, args.steps), args.warmup, peak)
    if ws == 1 and not args.no_cpu_baseline:
        from oracle.cpu_baseline import time_cpu_baseline

        sample = {"c1": 1024, "c2": 2048, "c3": 1024, "c4": 2048, "c5": 2048}[name]
        wl_cpu = workloads.make_workload(name, n=sample)
        cb = time_cpu_baseline(wl_cpu, sample, steps=3, warmup=1)
        line["cpu_baseline"] = {"value": cb["value"], "unit": UNIT, "cores": cb["cores"], "kind": "port",
                                "sample": cb["sample"]}
    print(json.dumps(line), flush=True)
    return 0


def read_traffic(config: str, kernel: str, n_local: int):
    """DRAM bytes of one launch over ``n_local`` rows, from a committed ncu summary if one exists
    (``profiles/traffic.txt`` lines: ``<config> <kernel> <bytes_per_launch> <rows> <note>``, the bytes of a
    launch over ``rows`` rows; every term of the traffic but the small tables grows with the rows, so the
    figure is scaled to the rows this rank's launch processes)."""
    p = ROOT / "profiles" / "traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 4 and parts[0] == config and parts[1] == kernel:
            try:
                return float(parts[2]) * n_local / float(parts[3])
            except ValueError:
                return None
    return None


if __name__ == "__main__":
    sys.exit(main())
