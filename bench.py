"""Throughput benchmark of the forecast path (one JSON line on rank 0).

Workload (BASELINE.json metric / configs[2]): Chronos-2-shaped random-init checkpoint (768-d,
12 layers, 12 heads, d_ff 3072, patch 16, 21 quantiles), 256 seeded series per GPU of 8192 steps
(5 % NaN), horizon 1024. One step = one forecast of the batch. Synthetic data (seeded sine +
random walk + noise, lognormal scale); random-init weights; no hub access.

  value  series/s with inputs resident in HBM (tsfm_forecast_chronos2_device), device time from
         CUDA events on the launching stream, L2 flushed between steps, max over ranks.
  e2e    series/s through the host entry point tsfm_forecast_chronos2 with pinned host buffers:
         H2D of the inputs and D2H of the quantiles inside the timed region.
  roofline  of the dominant kernel (the tcgen05 linear kernel): algorithmic FLOPs / summed
         CUDA-event launch time, against the measured sustained BF16 peak.
  cpu_baseline  the CPU restatement (oracle) on a bounded sample of the same workload.

`--impl reference` times the reference algorithm's CPU implementation instead (the oracle port,
all host threads; the Zig reference cannot be built on these hosts) on rank 0 only.

Multi-GPU: `python -m torch.distributed.run --nproc-per-node N bench.py --gpus N`: each rank
forecasts its own 256 series (weak scaling, no collective on the data path).
"""
import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(ROOT, "tsfm-zig_b200"), ROOT]

METRIC = "forecast series/sec at 1/2/4/8 B200 (Chronos-2-shaped ctx8192 H1024); % TC peak"
SERIES_PER_GPU = 256
CONTEXT = 8192
HORIZON = 1024
GF_PER_SERIES = 130.02  # algorithmic GFLOP per series at ctx 8192, H 1024 (2 FLOPs per MAC)


def series_seed(rank, b):
    """First generator seed of a rank's b series: ranks draw disjoint seeded blocks (weak scaling)."""
    return 1000 + rank * b


def max_over_ranks(x, world, device):
    """The slowest rank's figure: an all-reduce MAX over the job (x itself when world == 1)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--compute", default="f16c", choices=["f16c", "f16", "bf16"],
                    help="operand mode of the headline (f16c: FP16 + FP8 correction products, the mode that "
                         "meets the 1e-2 * sigma bound at this shape)")
    ap.add_argument("--no-compare", action="store_true",
                    help="skip the extra measurement of plain FP16 operands beside the headline")
    ap.add_argument("--series", type=int, default=SERIES_PER_GPU)
    ap.add_argument("--cpu-sample", type=int, default=4,
                    help="series timed on the CPU baseline leg (bolt-*/timestral: 0 skips it, for profiling captures)")
    ap.add_argument("--batch", type=int, default=None,
                    help="series of the bolt-*/timestral workloads (default: the BASELINE.json config's batch; "
                         "smaller batches are for profiling captures)")
    ap.add_argument("--csv-series", type=int, default=8192, help="series of the csv workload")
    ap.add_argument("--gemm-controls", action="store_true",
                    help="gemm workload: also time the weight-term-only corrected product and a plain FP16 product "
                         "with K doubled")
    ap.add_argument("--gemm-rows", type=int, default=256 * 577,
                    help="rows M of the gemm workload (default: the headline's 256 series x 577 tokens; smaller for "
                         "profiling captures)")
    ap.add_argument("--workload", default="chronos2",
                    choices=["chronos2", "bolt-small", "bolt-base", "timestral", "sweep", "csv", "parse",
                             "attention", "gemm", "seam"],
                    help="chronos2 is the headline; bolt-*/timestral are BASELINE.json's other configs, timed "
                         "through the host entry points (copies included); sweep is its Chronos-2 throughput sweep "
                         "(batch x context, one JSON line per point); csv renders the CLI's CSV output of an "
                         "8192-series, horizon-1024, 21-level forecast; parse reads an 8192-series x 8192-step "
                         "series file")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["bf16_tflops"], p["bf16_tflops_sustained"], p["hbm_gbs"], "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


class Clocks:
    """Samples nvidia-smi clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu, self.rows, self.proc = gpu, [], None
        self.window = (0.0, 0.0)

    def start(self):
        """Starts sampling every 50 ms (nvidia-smi needs a moment before its first line, so this
        runs before the warm-up); only the samples inside mark_begin() .. mark_end() count."""
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def mark_begin(self):
        self.window = (time.perf_counter(), float("inf"))

    def mark_end(self):
        self.window = (self.window[0], time.perf_counter())

    def __enter__(self):
        return self.start()

    def _read(self):
        for line in self.proc.stdout:
            now = time.perf_counter()
            if self.window[0] <= now <= self.window[1]:
                self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.t.join(timeout=2)

    def summary(self):
        sm = [float(r[1]) for r in self.rows if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            if len(r) >= 9:
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def build_model(devices, compute):
    from tsfm_b200 import Model
    from tsfm_spec import synthetic as syn
    cfg = syn.chronos2_config(context_length=CONTEXT, max_output_patches=64)
    w = syn.random_checkpoint(cfg, seed=20261201)
    return cfg, w, Model(cfg, w, devices=tuple(devices), compute=compute)


def traffic_from_profile():
    """DRAM bytes per GEMM launch (averaged over a whole forecast step, like `achieved`) from the
    committed ncu summary, if present."""
    p = os.path.join(ROOT, "profiles", "linear_tc_chronos2.md")
    try:
        for line in open(p):
            if line.startswith("traffic_bytes_per_gemm_launch:"):
                return float(line.split(":")[1])
    except Exception:
        pass
    return None


def cpu_baseline(sample):
    """The oracle (CPU restatement of the reference path) on `sample` series of the workload."""
    from oracle import binding as ob
    from tsfm_spec import config as cm, synthetic as syn
    from tsfm_spec.table import tensor_table
    cfg = syn.chronos2_config(context_length=CONTEXT, max_output_patches=64)
    w = syn.random_checkpoint(cfg, seed=20261201)
    m = ob.OracleModel(cm.parse(cfg), w, tensor_table)
    x = syn.seeded_series(sample, CONTEXT, seed=series_seed(0, SERIES_PER_GPU))  # the GPU arm's first series
    t0 = time.perf_counter()
    m.forecast_chronos2(x, HORIZON)
    dt = time.perf_counter() - t0
    return sample / dt, ob.get_threads(), dt


def run_reference(a, rank):
    if rank != 0:
        return
    # The oracle and the pure-Python formats only: nothing of the CUDA backend is loaded here.
    from oracle import binding as ob
    from tsfm_spec import config as cm, synthetic as syn
    from tsfm_spec.table import tensor_table
    ob.set_threads(os.cpu_count() or 1)
    cfg = syn.chronos2_config(context_length=CONTEXT, max_output_patches=64)
    w = syn.random_checkpoint(cfg, seed=20261201)
    m = ob.OracleModel(cm.parse(cfg), w, tensor_table)
    n = max(1, a.cpu_sample)
    x = syn.seeded_series(n, CONTEXT, seed=series_seed(0, SERIES_PER_GPU))  # the GPU arm's first series
    for _ in range(max(0, min(a.warmup, 1))):
        m.forecast_chronos2(x[:1], HORIZON)
    times = []
    for _ in range(a.steps):
        t0 = time.perf_counter()
        m.forecast_chronos2(x, HORIZON)
        times.append(time.perf_counter() - t0)
    ms = float(np.mean(times)) * 1e3
    v = n / (ms / 1e3)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "series/s", "n_gpus": a.gpus, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": "chronos2-ctx8192-h1024", "series_per_step": n, "context": CONTEXT,
                   "horizon": HORIZON, "l2": "n/a (CPU)"},
        "cpu_baseline": {"value": v, "unit": "series/s", "cores": ob.get_threads(), "kind": "port",
                         "sample": f"{n} series x 8192 steps, horizon 1024, per step"},
        "e2e": {"value": v, "unit": "series/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# Algorithmic GFLOP per series of the Chronos-2-shaped model at horizon 1024, by context length.
GF_BY_CONTEXT = {512: 20.53, 2048: 41.07, 8192: 130.02}


def run_sweep(a):
    """BASELINE.json's throughput sweep on the Chronos-2-shaped model: batch {1, 16, 256, 2048, 8192}
    x context {512, 2048, 8192}, horizon 1024, one GPU. Per point: device-resident series/s (CUDA events
    around each forecast, L2 flushed in between) and end-to-end series/s through the host entry point
    (pinned buffers, copies included), with the fraction of the measured burst BF16 peak."""
    import torch
    from tsfm_b200 import synthetic as syn
    burst = peaks()[0]
    cfg, w, model = build_model(0)
    del w
    q = 21
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda")
    stream = torch.cuda.current_stream()
    for ctx in (512, 2048, 8192):
        for b in (1, 16, 256, 2048, 8192):
            x = syn.seeded_series(b, ctx, seed=5000 + b)
            xd = torch.from_numpy(x).cuda()
            out = torch.empty((b, HORIZON, q), device="cuda")
            step = lambda: model.forecast_chronos2_device(xd.data_ptr(), b, ctx, HORIZON, out.data_ptr(),
                                                          stream.cuda_stream)
            for _ in range(max(3, a.warmup)):
                step()
            torch.cuda.synchronize()
            # About half a second of timed forecasts per point (at least 3).
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            step()
            e1.record(stream)
            e1.synchronize()
            est = max(e0.elapsed_time(e1), 1e-3)
            reps = int(min(50, max(3, 500.0 / est)))
            total = 0.0
            for _ in range(reps):
                flush.zero_()
                e0.record(stream)
                step()
                e1.record(stream)
                e1.synchronize()
                total += e0.elapsed_time(e1)
            ms = total / reps
            xp = torch.from_numpy(x).pin_memory().numpy()
            op = torch.empty((b, HORIZON, q), dtype=torch.float32).pin_memory().numpy()
            for _ in range(2):  # the second call captures the CUDA graphs that later calls replay
                model.forecast_chronos2(xp, HORIZON, out=op)
            t0 = time.perf_counter()
            for _ in range(reps):
                model.forecast_chronos2(xp, HORIZON, out=op)
            e2e_ms = (time.perf_counter() - t0) / reps * 1e3
            gf = GF_BY_CONTEXT[ctx]
            print(json.dumps({"workload": "sweep", "batch": b, "context": ctx, "horizon": HORIZON, "n_gpus": 1,
                              "ms_per_forecast": ms, "series_per_s": b / (ms / 1e3),
                              "e2e_ms_per_forecast": e2e_ms, "e2e_series_per_s": b / (e2e_ms / 1e3),
                              "tc_peak_frac": gf * 1e9 * b / (ms / 1e3) / (burst * 1e12), "steps": reps,
                              "gpu_launches_per_forecast": model.last_launch_count()}), flush=True)
            del xd, out
    model.close()


def run_family_workload(a):
    """BASELINE.json's Chronos-Bolt and Timestral configs on one GPU, through the host entry points
    (pinned inputs, host->device and device->host copies inside the timed region). Operand modes:
    the ones the parity tests hold at these shapes (Bolt: plain FP16, 1.6e-3 sigma at Bolt-base;
    Timestral: the corrected products, its configs[3] checkpoint in BF16 as BASELINE.json names it)."""
    import torch
    from tsfm_b200 import Model, covariates, synthetic as syn, timestral_options
    if a.workload == "bolt-small":
        cfg = syn.bolt_config()
        b, horizon, ctx = 64, 64, 2048
    elif a.workload == "bolt-base":
        cfg = syn.bolt_config(d_model=768, d_ff=3072, num_heads=12, num_layers=12)
        b, horizon, ctx = 4096, 256, 2048
    else:
        cfg = syn.timestral_config(d_model=1024, num_heads=16, mlp_hidden_dim=4096, num_layers=16, patch=32,
                                   context_length=4096, block_size=32)
        b, horizon, ctx = 128, 512, 4096
    if a.batch:
        b = a.batch
    ts = not a.workload.startswith("bolt")
    compute = "f16c" if ts else "f16"
    w = syn.random_checkpoint(cfg, seed=20261201, dtype="bf16" if ts else np.float32)
    model = Model(cfg, w, compute=compute)
    if a.workload.startswith("bolt"):
        x = torch.from_numpy(syn.seeded_series(b, ctx, seed=2000)).pin_memory().numpy()
        out = torch.empty((b, horizon, 9), dtype=torch.float32).pin_memory().numpy()
        run = lambda: model.forecast_bolt(x, horizon, out=out)
        h2d, d2h = x.nbytes, out.nbytes
    else:
        v = 8
        xs = syn.seeded_series(b * v, ctx, seed=3000).reshape(b, v, ctx)
        past = syn.ar1_covariates(b, 2, ctx, seed=31)
        known = syn.ar1_covariates(b, 1, ctx + horizon, seed=32)
        cov = covariates(past=past, known=known)
        opts = timestral_options()
        out = np.empty((b, v, horizon, 9), np.float32)
        run = lambda: model.forecast_timestral(xs, horizon, cov=cov, opts=opts, out=out)
        h2d = xs.size * 5 + past.nbytes + known.nbytes
        d2h = out.nbytes
    for _ in range(max(1, min(a.warmup, 2))):
        run()
    torch.cuda.synchronize()
    steps = max(1, min(a.steps, 3))
    t0 = time.perf_counter()
    for _ in range(steps):
        run()
    torch.cuda.synchronize()
    ms = (time.perf_counter() - t0) / steps * 1e3
    # Per-kernel-class device time on one separate, untimed forecast.
    model.profile(True)
    model.profile_reset()
    run()
    torch.cuda.synchronize()
    cls = {c: model.profile_read(c) for c in ("gemm", "attention", "rmsnorm", "patch", "head", "other")}
    model.profile(False)
    kernels = {c: {"launches": v["launches"], "ms": v["ms"]} for c, v in cls.items() if v["launches"]}
    # CPU baseline: the oracle (the reference algorithm restated, all host threads) on a bounded
    # sample of the same workload (skipped with --cpu-sample 0, for profiling captures).
    if a.cpu_sample == 0:
        line = {"workload": a.workload, "series": b, "ms_per_step": ms, "value": b / (ms / 1e3), "unit": "series/s",
                "gpu_launches": model.last_launch_count(), "kernels": kernels, "cpu_baseline": None}
        print(json.dumps(line), flush=True)
        model.close()
        return
    from oracle import binding as ob
    from tsfm_spec import config as cm
    from tsfm_spec.table import tensor_table
    ob.set_threads(os.cpu_count() or 1)
    om = ob.OracleModel(cm.parse(cfg), w, tensor_table)
    if a.workload.startswith("bolt"):
        ns = 16 if a.workload == "bolt-small" else 2
        t0 = time.perf_counter()
        om.forecast_bolt(x[:ns], horizon)
    else:
        ns = 1
        sub_cov = covariates(past=past[:ns], known=known[:ns])
        t0 = time.perf_counter()
        om.forecast_timestral(xs[:ns], np.isfinite(xs[:ns]), horizon, cov=sub_cov[0], opts=opts)
    cpu_dt = time.perf_counter() - t0
    del om, w
    line = {"metric": f"forecast series/sec ({a.workload}, BASELINE.json config)", "value": b / (ms / 1e3),
            "unit": "series/s", "n_gpus": 1, "steps": steps, "ms_per_step": ms, "higher_is_better": True,
            "dtype": "f16+f8 (FP16 operands plus FP8 correction products)" if ts else "f16",
            "data": "synthetic (seeded series, random-init N(0,0.02) weights" + (", BF16 checkpoint)" if ts else ")"),
            "config": {"workload": a.workload, "series": b, "context": ctx, "horizon": horizon, "compute": compute,
                       "checkpoint": "bf16" if ts else "f32",
                       "timing": "host entry point, pinned buffers, copies included"},
            "e2e": {"value": b / (ms / 1e3), "unit": "series/s", "h2d_bytes_per_step": int(h2d),
                    "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": model.last_launch_count(), "kernels": kernels,
            "cpu_baseline": {"value": ns / cpu_dt, "unit": "series/s", "cores": ob.get_threads(), "kind": "port",
                             "sample": f"{ns} series of the same workload (oracle restatement)"}}
    print(json.dumps(line), flush=True)
    model.close()


def forecast_like_values(series, horizon, q, seed):
    """Quantile forecasts shaped like the models' output: a per-series level and scale, a random
    walk over the horizon and increasing quantile offsets, in float32 (full-precision digits)."""
    rng = np.random.default_rng(seed)
    level = rng.lognormal(3.0, 2.0, size=(series, 1, 1, 1))
    walk = np.cumsum(rng.standard_normal((series, 1, horizon, 1)), axis=2) * 0.05
    offs = np.sort(rng.standard_normal((series, 1, horizon, q)), axis=3)
    return (level * (1.0 + walk + 0.1 * offs)).astype(np.float32)


def run_csv(a):
    """The CLI's CSV output (writeCsv, src/main.zig:181-198) of an 8192-series, horizon-1024,
    21-level forecast on one GPU: 176 M numbers. value: series/s with the forecast resident in HBM
    (tsfm_csv_format_device, CUDA events); e2e: series/s through tsfm_csv_format from pinned host
    values into a pinned host text buffer (copies both ways inside the timed region)."""
    import ctypes
    import torch
    import tsfm_b200 as tb
    from tsfm_b200 import csv
    series, horizon, q = a.csv_series, 1024, 21
    levels = np.array([0.01, 0.05] + [round(0.05 * i, 2) for i in range(2, 19)] + [0.95, 0.99], np.float64)
    assert levels.size == q
    vals = forecast_like_values(series, horizon, q, seed=77)
    stream = torch.cuda.current_stream()
    dv = torch.from_numpy(vals).cuda()
    need = ctypes.c_size_t(0)
    tb.lib.tsfm_csv_format_device(dv.data_ptr(), series, 1, horizon, levels.ctypes.data, q, None, 0,
                                  ctypes.byref(need), stream.cuda_stream)
    text_bytes = need.value
    dout = torch.empty(text_bytes, dtype=torch.uint8, device="cuda")
    run_dev = lambda: csv.format_csv_device(dv.data_ptr(), series, 1, horizon, levels, dout.data_ptr(),
                                            text_bytes, stream.cuda_stream)
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda")
    for _ in range(max(3, a.warmup)):
        run_dev()
    torch.cuda.synchronize()
    steps = max(3, a.steps)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    csv.profile(True)
    total = 0.0
    with Clocks(0) as clocks:
        time.sleep(0.3)
        clocks.mark_begin()
        for _ in range(steps):
            flush.zero_()
            e0.record(stream)
            run_dev()
            e1.record(stream)
            e1.synchronize()
            total += e0.elapsed_time(e1)
        clocks.mark_end()
    kern = {k: csv.profile_read(k) for k in ("describe", "scan", "text")}
    csv.profile(False)
    ms = total / steps
    # e2e: pinned host values in, pinned host text out.
    hv = torch.from_numpy(vals).pin_memory()
    hout = torch.empty(text_bytes, dtype=torch.uint8).pin_memory()
    n = ctypes.c_size_t(0)
    run_host = lambda: tb.check(tb.lib.tsfm_csv_format(hv.data_ptr(), series, 1, horizon, levels.ctypes.data, q, 0,
                                                       hout.data_ptr(), text_bytes, ctypes.byref(n)))
    for _ in range(2):
        run_host()
    t0 = time.perf_counter()
    for _ in range(steps):
        run_host()
    e2e_ms = (time.perf_counter() - t0) / steps * 1e3
    clk = clocks.summary()
    # Roofline of the CSV kernels together: the algorithm reads each value once (4 bytes) and
    # writes its text once; the packed digits between the passes are not counted.
    hbm_burst = peaks()[2]
    kern_ms = sum(v["ms"] for v in kern.values()) / steps
    alg = vals.nbytes + text_bytes
    achieved = alg / (kern_ms / 1e3) / 1e9
    # CPU baseline: the oracle's writeCsv restatement (all host threads) on 256 series.
    from oracle import binding as ob
    sample = vals[:256]
    t0 = time.perf_counter()
    ob.csv_format(sample, levels)
    cpu_dt = time.perf_counter() - t0
    line = {"metric": f"CSV output series/sec (writeCsv of a {series}-series H1024 21-level forecast)",
            "value": series / (ms / 1e3), "unit": "series/s", "n_gpus": 1, "steps": steps, "warmup": a.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic (seeded quantile forecasts, float32)",
            "config": {"workload": "csv", "series": series, "horizon": horizon, "levels": q,
                       "text_bytes": text_bytes, "l2": "flushed between steps (256 MiB write)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_burst, "unit": "GB/s",
                         "frac": achieved / hbm_burst, "traffic": None,
                         "kernel": "csv_describe + csv_scan + csv_text (summed CUDA-event time)",
                         "algorithmic_bytes": alg},
            "kernels": kern,
            "cpu_baseline": {"value": 256 / cpu_dt, "unit": "series/s", "cores": ob.get_threads(), "kind": "port",
                             "sample": "256 series x 1024 steps x 21 levels (oracle writeCsv restatement)"},
            "e2e": {"value": series / (e2e_ms / 1e3), "unit": "series/s", "h2d_bytes_per_step": int(vals.nbytes),
                    "d2h_bytes_per_step": int(text_bytes)},
            "gpu_launches": sum(v["launches"] for v in kern.values()) // steps,
            "clocks": clk}
    print(json.dumps(line), flush=True)


def run_parse(a):
    """The reader's parseBlocks (core/series.zig:21-68) of a series file with 8192 series of 8192
    steps, one series per comma-separated line (5 % empty tokens = missing). value: series/s with
    the text resident in HBM (tsfm_parse_blocks_device to f32, as the forecast consumes it);
    e2e: series/s through tsfm_parse_blocks from pinned host text to pinned host f64 values."""
    import ctypes
    import torch
    import tsfm_b200 as tb
    from tsfm_b200 import synthetic as syn
    series, steps = a.csv_series, CONTEXT
    # 256 distinct seeded series, repeated to the full count (every line is still parsed).
    base = syn.seeded_series(256, steps, seed=4242)
    lines = [",".join("" if np.isnan(v) else repr(float(v)) for v in row).encode() for row in base]
    text = b"\n".join(lines[i % 256] for i in range(series)) + b"\n"
    n = len(text)
    stream = torch.cuda.current_stream()
    dt = torch.from_numpy(np.frombuffer(text, np.uint8).copy()).cuda()
    out32 = torch.empty(series * steps, dtype=torch.float32, device="cuda")
    b, r, l = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_size_t()
    run_dev = lambda: tb.check(tb.lib.tsfm_parse_blocks_device(dt.data_ptr(), n, None, out32.data_ptr(),
                                                               out32.numel(), ctypes.byref(b), ctypes.byref(r),
                                                               ctypes.byref(l), stream.cuda_stream))
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda")
    for _ in range(max(3, a.warmup)):
        run_dev()
    assert (b.value, r.value, l.value) == (1, series, steps)
    steps_t = max(3, a.steps)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    total = 0.0
    with Clocks(0) as clocks:
        time.sleep(0.3)
        clocks.mark_begin()
        for _ in range(steps_t):
            flush.zero_()
            e0.record(stream)
            run_dev()
            e1.record(stream)
            e1.synchronize()
            total += e0.elapsed_time(e1)
        clocks.mark_end()
    ms = total / steps_t
    ht = torch.from_numpy(np.frombuffer(text, np.uint8).copy()).pin_memory()
    hv = torch.empty(series * steps, dtype=torch.float64).pin_memory()
    run_host = lambda: tb.check(tb.lib.tsfm_parse_blocks(ht.data_ptr(), n, 0, hv.data_ptr(), hv.numel(),
                                                         ctypes.byref(b), ctypes.byref(r), ctypes.byref(l)))
    for _ in range(2):
        run_host()
    t0 = time.perf_counter()
    for _ in range(steps_t):
        run_host()
    e2e_ms = (time.perf_counter() - t0) / steps_t * 1e3
    # CPU baseline: the oracle's parseBlocks restatement (one thread, as the reference) on 64 series.
    from oracle import binding as ob
    sample = b"\n".join(lines[:64]) + b"\n"
    vals = np.zeros(64 * steps + 16, np.float64)
    t0 = time.perf_counter()
    ob.lib.oracle_parse_blocks(sample, vals.ctypes.data, vals.size, ctypes.byref(b), ctypes.byref(r),
                               ctypes.byref(l))
    cpu_dt = time.perf_counter() - t0
    hbm_burst = peaks()[2]
    alg = n + series * steps * 4  # text read once, f32 values written once
    achieved = alg / (ms / 1e3) / 1e9
    line = {"metric": f"series file parse series/sec ({series} series x {steps} steps, parseBlocks)",
            "value": series / (ms / 1e3), "unit": "series/s", "n_gpus": 1, "steps": steps_t, "warmup": a.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (seeded series, Python repr of float32 values, 5 % empty)",
            "config": {"workload": "parse", "series": series, "steps": steps, "text_bytes": n,
                       "l2": "flushed between steps (256 MiB write)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_burst, "unit": "GB/s",
                         "frac": achieved / hbm_burst, "traffic": None,
                         "kernel": "whole reader (6 kernels, CUDA events around the call)", "algorithmic_bytes": alg},
            "cpu_baseline": {"value": 64 / cpu_dt, "unit": "series/s", "cores": 1, "kind": "port",
                             "sample": f"64 series x {steps} steps (oracle parseBlocks restatement, strtod)"},
            "e2e": {"value": series / (e2e_ms / 1e3), "unit": "series/s", "h2d_bytes_per_step": n,
                    "d2h_bytes_per_step": series * steps * 8},
            "gpu_launches": 6, "clocks": clocks.summary()}
    print(json.dumps(line), flush=True)


def run_attention(a):
    """The self-attention kernel alone at the families' shapes (tsfm_kernel_attention, CUDA events,
    L2 flushed between launches): Chronos-2 (256 sequences of 577 tokens, 12 heads, key-validity
    mask), Chronos-Bolt-base (4096 sequences of 129 tokens, 12 heads, relative-position bias) and
    Timestral (2816 rows of 160 tokens, 16 heads, causal over valid keys). TFLOP/s counts
    4 * n^2 * 64 per (sequence, head), halved for the causal mask: the useful work only."""
    import torch
    import tsfm_b200 as tb
    stream = torch.cuda.current_stream()
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda")
    burst = peaks()[0]
    shapes = (("chronos2", 256, 577, 12, False, 0), ("bolt-base", a.csv_series // 2, 129, 12, True, 0),
              ("timestral", 2816 * a.csv_series // 8192, 160, 16, False, 1))
    for name, G, n, heads, rel, mode in shapes:
        g = torch.Generator(device="cuda").manual_seed(7)
        ld = 3 * heads * 64
        qkv = (torch.randn(G * n, ld, device="cuda", generator=g) * 0.5).half()
        kv = (torch.rand(G, n, device="cuda", generator=g) > 0.05).to(torch.uint8)
        relb = torch.randn(heads, 2 * n - 1, device="cuda", generator=g) if rel else None
        o = torch.empty(G * n, heads * 64, device="cuda", dtype=torch.float16)
        run = lambda: tb.check(tb.lib.tsfm_kernel_attention(
            qkv.data_ptr(), qkv.data_ptr() + heads * 64 * 2, qkv.data_ptr() + 2 * heads * 64 * 2, ld, o.data_ptr(),
            heads * 64, kv.data_ptr(), None if relb is None else relb.data_ptr(), G, heads, n, 0.125, mode, 1,
            stream.cuda_stream))
        for _ in range(max(3, a.warmup)):
            run()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        total, steps = 0.0, max(3, a.steps)
        for _ in range(steps):
            flush.zero_()
            e0.record(stream)
            run()
            e1.record(stream)
            e1.synchronize()
            total += e0.elapsed_time(e1)
        ms = total / steps
        tf = 4.0 * n * n * 64 * heads * G / (ms / 1e3) / 1e12 / (2.0 if mode == 1 else 1.0)
        print(json.dumps({"workload": "attention", "shape": name, "sequences": G, "tokens": n, "heads": heads,
                          "rel_bias": rel, "mask_mode": mode, "ms": ms, "tflops": tf, "tc_peak_frac": tf / burst,
                          "us_per_sequence_head": ms * 1e3 / (G * heads)}), flush=True)
        del qkv, o


def run_gemm(a):
    """The encoder's linear layers alone at the Chronos-2 headline shape (M = 256 x 577 = 147,712
    rows): qkv (2304 x 768, FP16 out), o and the folded group projection (768 x 768, FP32
    accumulate), wi (3072 x 768, ReLU, FP16 out), wo (768 x 3072, FP32 accumulate), each with plain
    FP16 operands (tsfm_kernel_linear) and as the corrected product (tsfm_kernel_linear_f16c with the
    FP8 companions; wi's FP16 output with its companion, as the forward writes it). CUDA events per
    launch, L2 flushed between launches; TFLOP/s = 2 M N K / time (the algorithmic work; the
    corrected product executes twice the tensor-core work)."""
    import ctypes
    import torch
    import tsfm_b200 as tb
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda")
    burst = peaks()[0]
    M = a.gemm_rows
    g = torch.Generator(device="cuda").manual_seed(3)
    shapes = (("qkv", 2304, 768, 0, 0), ("o", 768, 768, 2, 0), ("wi", 3072, 768, 0, 1), ("wo", 768, 3072, 2, 0))
    for name, N, K, out_mode, act in shapes:
        x = torch.randn(M, K, device="cuda", generator=g)
        w = torch.randn(N, K, device="cuda", generator=g) * 0.02
        x16, w16 = x.half(), w.half()
        xc16 = torch.empty(M, K, device="cuda", dtype=torch.float16)
        x8 = torch.empty(M, 2 * K, device="cuda", dtype=torch.uint8)
        wc16 = torch.empty(N, K, device="cuda", dtype=torch.float16)
        w8 = torch.empty(N, 2 * K, device="cuda", dtype=torch.uint8)
        scale = ctypes.c_float(0.0)
        tb.check(tb.lib.tsfm_kernel_split_f16c(x.data_ptr(), M, K, xc16.data_ptr(), x8.data_ptr(), sp))
        tb.check(tb.lib.tsfm_kernel_weight_f16c(w.data_ptr(), N, K, wc16.data_ptr(), w8.data_ptr(), ctypes.byref(scale),
                                                sp))
        del x, w
        y = torch.zeros(M, N, device="cuda", dtype=torch.float16 if out_mode == 0 else torch.float32)
        # The forward writes an FP8 companion only where the output feeds a corrected product: the
        # MLP hidden (wi -> wo); qkv feeds the attention, which reads FP16.
        y8 = torch.empty(M, 2 * N, device="cuda", dtype=torch.uint8) if name == "wi" else None
        runs = {
            "f16": lambda: tb.check(tb.lib.tsfm_kernel_linear(x16.data_ptr(), 1, w16.data_ptr(), 1, None, y.data_ptr(),
                                                              out_mode, act, M, N, K, K, K, N, sp)),
            "f16c": lambda: tb.check(tb.lib.tsfm_kernel_linear_f16c(
                xc16.data_ptr(), x8.data_ptr(), wc16.data_ptr(), w8.data_ptr(), scale.value, None, y.data_ptr(),
                None if y8 is None else y8.data_ptr(), out_mode, act, M, N, K, 2, sp)),
        }
        if a.gemm_controls:
            # Controls: the weight term only (x_hi (W - f16(W)): 1.5x the FP16 stages), and a plain FP16
            # product with K doubled (the corrected product's stage count, every stage FP16).
            x2 = torch.randn(M, 2 * K, device="cuda", generator=g).half()
            w2 = (torch.randn(N, 2 * K, device="cuda", generator=g) * 0.02).half()
            runs["f16c-weight-term"] = lambda: tb.check(tb.lib.tsfm_kernel_linear_f16c(
                xc16.data_ptr(), x8.data_ptr(), wc16.data_ptr(), w8.data_ptr(), scale.value, None, y.data_ptr(),
                None if y8 is None else y8.data_ptr(), out_mode, act, M, N, K, 1, sp))
            runs["f16-2k"] = lambda: tb.check(tb.lib.tsfm_kernel_linear(
                x2.data_ptr(), 1, w2.data_ptr(), 1, None, y.data_ptr(), out_mode, act, M, N, 2 * K, 2 * K, 2 * K, N, sp))
            if y8 is not None:  # wi without writing its output's companion
                runs["f16c-no-companion"] = lambda: tb.check(tb.lib.tsfm_kernel_linear_f16c(
                    xc16.data_ptr(), x8.data_ptr(), wc16.data_ptr(), w8.data_ptr(), scale.value, None, y.data_ptr(),
                    None, out_mode, act, M, N, K, 2, sp))
        for mode, run in runs.items():
            for _ in range(max(3, a.warmup)):
                run()
            torch.cuda.synchronize()
            total, steps = 0.0, max(3, a.steps)
            for _ in range(steps):
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                run()
                e1.record(stream)
                e1.synchronize()
                total += e0.elapsed_time(e1)
            ms = total / steps
            tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
            work = {"f16": 1.0, "f16c": 2.0, "f16c-weight-term": 1.5, "f16-2k": 2.0, "f16c-no-companion": 2.0}[mode]
            print(json.dumps({"workload": "gemm", "shape": name, "mode": mode, "M": M, "N": N, "K": K, "ms": ms,
                              "tflops": tf, "tensor_tflops_executed": tf * work,
                              "frac_of_burst": tf / burst}), flush=True)
        del x16, w16, xc16, x8, wc16, w8, y, y8


SEAM_SHAPES = (("qkv", 2304, 768), ("o", 768, 768), ("wi", 3072, 768), ("wo", 768, 3072))


def run_seam(a, reference=False):
    """The reference's GEMM seam (platform/cuda/gemm.c:232-330): C[m, n] = A[m, k] W[n, k]^T with
    host operands (pinned), W registered once (cuda_weight_register / tsfm_weight_register, as
    nn.linear does), on the Chronos-2 linear shapes at M = 147,712 rows; one JSON line per shape
    with the wall time per call (copies included: the call returns when C is on the host) and the
    error against float64 on 256 sampled rows. This arm: tsfm_sgemm_nt (split-TF32 on the tcgen05
    kernel); `--impl reference`: the reference's own gemm.c compiled from its source
    (oracle/_ref/libgemm_ref.so, cuBLAS SGEMM)."""
    import ctypes
    import torch
    if reference:
        # gemm.c dlopens cuBLAS from TSFM_CUDA_LIB_DIR (its documented setting). Point it at the
        # cuBLAS that torch has already loaded: a second cuBLAS build would bind its DT_NEEDED
        # cuBLASLt by soname to torch's copy and fail to load.
        if "TSFM_CUDA_LIB_DIR" not in os.environ:
            import nvidia.cublas
            os.environ["TSFM_CUDA_LIB_DIR"] = os.path.join(list(nvidia.cublas.__path__)[0], "lib")
        lib = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libgemm_ref.so"))
        reg, nt = lib.cuda_weight_register, lib.cuda_sgemm_nt
    else:
        import tsfm_b200 as tb
        reg, nt = tb.lib.tsfm_weight_register, tb.lib.tsfm_sgemm_nt
    reg.restype, reg.argtypes = ctypes.c_void_p, [ctypes.c_void_p, ctypes.c_size_t]
    nt.restype = ctypes.c_int
    nt.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    M = a.gemm_rows
    rng = np.random.default_rng(9)
    for name, N, K in SEAM_SHAPES:
        A = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).pin_memory()
        W = (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float32)
        C = torch.empty((M, N), dtype=torch.float32).pin_memory()
        h = reg(W.ctypes.data, W.size)
        if not h:
            print(json.dumps({"workload": "seam", "shape": name, "failed": "weight registration"}), flush=True)
            continue
        call = lambda: nt(M, N, K, 1.0, A.data_ptr(), K, None, K, C.data_ptr(), N, h)  # noqa: E731
        st = call()
        for _ in range(max(0, a.warmup - 1)):
            st = st or call()
        times = []
        for _ in range(max(1, min(a.steps, 5))):
            t0 = time.perf_counter()
            st = st or call()
            times.append(time.perf_counter() - t0)
        rows = rng.choice(M, 256, replace=False)
        ref = A.numpy()[rows].astype(np.float64) @ W.astype(np.float64).T
        mag = np.abs(A.numpy()[rows]).astype(np.float64) @ np.abs(W).astype(np.float64).T
        err = float(np.max(np.abs(C.numpy()[rows] - ref) / mag))
        ms = float(np.median(times)) * 1e3
        line = {"workload": "seam", "impl": "reference" if reference else "b200", "shape": name, "M": M, "N": N,
                "K": K, "status": int(st), "ms_per_call": ms, "tflops": 2.0 * M * N * K / (ms / 1e3) / 1e12,
                "max_err_over_abs_products": err,
                "bytes_copied_per_call": (M * K + M * N) * 4, "what": "cuBLAS SGEMM via gemm.c" if reference
                else "split-TF32 tcgen05 (tsfm_sgemm_nt)"}
        print(json.dumps(line), flush=True)
        del A, C


def measure(model, a, x, world, barrier, clk=None):
    """One operand mode of the headline workload: device-resident series/s (CUDA events on the
    launching stream, L2 flushed between steps, max over ranks), end-to-end series/s through the
    host entry point (pinned buffers, copies inside the timed region), and per-kernel-class
    device times from separate, untimed steps."""
    import torch
    b, q = x.shape[0], 21
    xd = torch.from_numpy(x).cuda()
    out = torch.empty((b, HORIZON, q), device="cuda")
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda")
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream

    def step():
        model.forecast_chronos2_device(xd.data_ptr(), b, CONTEXT, HORIZON, out.data_ptr(), sp)

    for _ in range(max(3, a.warmup)):
        step()
    torch.cuda.synchronize()
    launches = model.last_launch_count()
    barrier()
    torch.cuda.synchronize()
    total_ms = 0.0
    if clk:
        clk.mark_begin()
    for _ in range(a.steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        step()
        e1.record(stream)
        e1.synchronize()
        total_ms += e0.elapsed_time(e1)
    if clk:
        clk.mark_end()
    torch.cuda.synchronize()
    barrier()
    ms_step = max_over_ranks(total_ms, world, "cuda") / a.steps
    value = b * world / (ms_step / 1e3)

    # End to end through the host entry point: pinned inputs in, quantiles out. Warm-up as above
    # (the second call with these buffers captures the CUDA graphs; later calls replay them).
    xp = torch.from_numpy(x).pin_memory()
    op = torch.empty((b, HORIZON, q), dtype=torch.float32).pin_memory()
    xnp, onp = xp.numpy(), op.numpy()
    for _ in range(max(3, a.warmup)):
        model.forecast_chronos2(xnp, HORIZON, out=onp)
    barrier()
    t0 = time.perf_counter()
    for _ in range(a.steps):
        model.forecast_chronos2(xnp, HORIZON, out=onp)
    e2e_s = (time.perf_counter() - t0) / a.steps
    barrier()
    e2e = b * world / max_over_ranks(e2e_s, world, "cuda")

    model.profile(True)
    model.profile_reset()
    for _ in range(2):
        step()
    torch.cuda.synchronize()
    cls = {c: model.profile_read(c) for c in ("gemm", "attention", "rmsnorm", "patch", "head", "other")}
    model.profile(False)
    g = cls["gemm"]
    achieved = g["work"] / (g["ms"] / 1e3) / 1e12 if g["ms"] > 0 else None
    kernels = {c: {"launches_per_step": v["launches"] / 2, "ms_per_step": v["ms"] / 2,
                   "share": v["ms"] / max(1e-9, sum(u["ms"] for u in cls.values()))} for c, v in cls.items()}
    if cls["attention"]["ms"] > 0:
        kernels["attention"]["tflops"] = cls["attention"]["work"] / (cls["attention"]["ms"] / 1e3) / 1e12
    # Memory-bound classes: algorithmic bytes (recorded per launch) over their device time, and the
    # fraction of the measured HBM copy bandwidth.
    for c in ("rmsnorm",):
        if cls[c]["ms"] > 0 and cls[c]["work"] > 0:
            kernels[c]["gbs"] = cls[c]["work"] / (cls[c]["ms"] / 1e3) / 1e9
            kernels[c]["hbm_frac"] = kernels[c]["gbs"] / peaks()[2]
    burst = peaks()[0]
    return {"value": value, "ms_per_step": ms_step, "e2e": e2e, "launches": launches, "kernels": kernels,
            "gemm_tflops": achieved, "tc_peak_frac": (GF_PER_SERIES * 1e9 * b / (ms_step / 1e3)) / (burst * 1e12)}


def library_multi_device(a, world):
    """The library's own multi-GPU path (rank 0 only, the other ranks waiting): one model with a
    replica on each of the job's `world` devices forecasts world x 256 series through the host
    entry point (strong scaling of one call: series sharded by the library, one host thread per
    device), timed by the wall clock around the blocking call; the result is compared bit for bit
    with a one-device model's."""
    from tsfm_spec import synthetic as syn
    _, w, multi = build_model(range(world), a.compute)
    b = a.series * world
    x = syn.seeded_series(b, CONTEXT, seed=series_seed(0, a.series))
    for _ in range(2):
        got = multi.forecast_chronos2(x, HORIZON)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        got = multi.forecast_chronos2(x, HORIZON)
    dt = (time.perf_counter() - t0) / a.steps
    multi.close()
    _, _, one = build_model([0], a.compute)
    ref = one.forecast_chronos2(x, HORIZON)
    t0 = time.perf_counter()
    ref = one.forecast_chronos2(x, HORIZON)
    dt1 = time.perf_counter() - t0
    one.close()
    del w
    return {"devices": world, "series_per_call": b, "e2e": b / dt, "e2e_one_device": b / dt1,
            "unit": "series/s", "bit_identical_to_one_device": bool(np.array_equal(got, ref)),
            "how": "one tsfm_model with a replica per device, host buffers, wall clock around the blocking call"}


def main():
    a = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        if a.workload == "seam":
            return run_seam(a, reference=True) if rank == 0 else None
        return run_reference(a, rank)
    if a.workload != "chronos2":
        if rank == 0:
            {"sweep": run_sweep, "csv": run_csv, "parse": run_parse, "attention": run_attention, "gemm": run_gemm,
             "seam": run_seam}.get(
                a.workload, run_family_workload)(a)
        return

    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    from tsfm_spec import synthetic as syn
    b = a.series
    x = syn.seeded_series(b, CONTEXT, seed=series_seed(rank, b))
    _, w, model = build_model([local], a.compute)
    del w
    clk = Clocks(local).start()
    head = measure(model, a, x, world, barrier, clk)
    clk.__exit__()
    model.close()
    fast = None
    if not a.no_compare and a.compute != "f16":
        _, w, m16 = build_model([local], "f16")
        del w
        fast = measure(m16, a, x, world, barrier)
        m16.close()
    multi = None
    if world > 1:
        # Rank 0 alone drives every GPU through one library model while the other ranks wait on the
        # host (a gloo barrier): no collective kernel sits on a GPU that rank 0's kernels use.
        host = dist.new_group(backend="gloo")
        torch.cuda.synchronize()
        dist.barrier(group=host)
        if rank == 0:
            try:
                multi = library_multi_device(a, world)
            except Exception as ex:  # reported, never hides the headline
                multi = {"failed": str(ex)}
        dist.barrier(group=host)

    if rank == 0:
        burst, sustained, hbm, src = peaks()
        cpu = None
        try:
            v, cores, dt = cpu_baseline(a.cpu_sample)
            cpu = {"value": v, "unit": "series/s", "cores": cores, "kind": "port",
                   "sample": f"{a.cpu_sample} series x 8192 steps, horizon 1024, the GPU arm's first series "
                             f"({dt:.1f} s)"}
        except Exception as ex:  # the baseline leg must not hide the GPU number
            cpu = {"value": None, "unit": "series/s", "cores": None, "kind": "port", "sample": f"failed: {ex}"}
        corr = a.compute == "f16c"
        achieved = head["gemm_tflops"]
        dtype = {"f16c": "f16+f8 (FP16 operands plus FP8 correction products, FP32 accumulation)",
                 "f16": "f16 (FP32 accumulation)", "bf16": "bf16 (FP32 accumulation)"}[a.compute]
        line = {
            "metric": METRIC, "value": head["value"], "unit": "series/s", "n_gpus": world, "steps": a.steps,
            "warmup": max(3, a.warmup), "ms_per_step": head["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": dtype,
            "data": "synthetic (seeded sine + random walk + noise, 5% NaN; random-init N(0,0.02) weights)",
            "config": {"workload": "chronos2-ctx8192-h1024", "compute": a.compute, "d_model": 768, "layers": 12,
                       "heads": 12, "d_ff": 3072, "patch": 16, "quantiles": 21, "series_per_gpu": b,
                       "global_batch": b * world, "context": CONTEXT, "horizon": HORIZON,
                       "parallelism": f"series-sharded x{world}", "l2": "flushed between steps (256 MB write)",
                       "parity": ("max |dq| <= 1e-2 * sigma at this shape (tests/test_chronos2_gpu.py)" if corr
                                  else "plain operands: the quantile tails exceed 1e-2 * sigma at this shape")},
            "tc_peak_frac": head["tc_peak_frac"],
            "roofline": {"bound": "tensor", "kernel": "linear_tc_kernel (tcgen05 GEMM)", "achieved": achieved,
                         "peak": sustained, "unit": "TFLOP/s", "frac": achieved / sustained if achieved else None,
                         "peak_source": f"{src} bf16_tflops_sustained", "traffic": traffic_from_profile(),
                         "tensor_work_per_algorithmic_flop": 2.0 if corr else 1.0},
            "kernels": head["kernels"],
            "cpu_baseline": cpu,
            "e2e": {"value": head["e2e"], "unit": "series/s", "h2d_bytes_per_step": b * CONTEXT * 4,
                    "d2h_bytes_per_step": b * HORIZON * 21 * 4},
            "gpu_launches": head["launches"] * a.steps,
            "clocks": clk.summary(),
        }
        if fast:
            line["f16_mode"] = {"value": fast["value"], "e2e": fast["e2e"], "ms_per_step": fast["ms_per_step"],
                                "tc_peak_frac": fast["tc_peak_frac"], "gemm_tflops": fast["gemm_tflops"],
                                "kernels": fast["kernels"],
                                "parity": "single-pass FP16 operands: quantile tails exceed 1e-2 * sigma here"}
        if multi:
            line["library_multi_gpu"] = multi
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
