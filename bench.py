"""Benchmark of the rapier_b200 decode hot path (driver contract: one JSON line from rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl rapier|reference] [--workload gemv|decode]

Workloads (synthetic seeded data, no model file):
  gemv    config 1: Q6_K x Q8_1 GEMV, W 12288x4096 ~ N(0, 0.02), x 4096 ~ N(0, 1), ncols 2 (the verify's
          shape). A step is one GEMV; weights rotate over 8 packed copies (330 MB > the 126 MB L2), so
          every step streams its weights from HBM.

Multi-GPU: one process per GPU under torchrun; each rank runs an independent replica of the workload
(the GEMV path has no exchange step), value = units of all ranks / max over ranks of the timed region.

--impl reference times the reference's CPU restatement (the oracle; the reference itself cannot be built
here, it needs the out-of-tree Strata/ggml headers and HIP) on the host cores, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HBM_FALLBACK_GBS = 6650.0


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK_GBS, "fallback"


# ------------------------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ------------------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                vals = [v.strip() for v in out.stdout.strip().split(",")]
                if len(vals) == 6:
                    self.samples.append(vals)
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[2 + i].strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


# ------------------------------------------------------------------------------------------------------
# distributed plumbing
# ------------------------------------------------------------------------------------------------------
def dist_init(n_gpus: int):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
        pg = dist
    return rank, world, local, pg


def max_over_ranks(x: float, pg, device) -> float:
    if pg is None:
        return x
    import torch

    t = torch.tensor([x], dtype=torch.float64, device=device)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def barrier(pg, device):
    import torch

    torch.cuda.synchronize(device)
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize(device)


# ------------------------------------------------------------------------------------------------------
# gemv workload (config 1)
# ------------------------------------------------------------------------------------------------------
GEMV_N_IN, GEMV_N_OUT, GEMV_NCOLS, GEMV_COPIES = 4096, 12288, 2, 8


def gemv_algorithmic_bytes(n_in, n_out, ncols):
    w = n_in // 256 * 210 * n_out
    return w + ncols * (n_in // 32 * 36) + ncols * n_out * 4


def run_gemv(args, rank, world, local, pg):
    import torch

    from oracle import oracle as O
    from rapier_b200 import ops

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(device=dev)  # the C-ABI requires an explicit (non-default) stream
    torch.cuda.set_stream(stream)
    n_in, n_out, nc = GEMV_N_IN, GEMV_N_OUT, GEMV_NCOLS
    wb = ops.native_mmvq_weight_bytes(14, n_in, n_out)
    # synthetic weights: seeded N(0, 0.02) quantized by the oracle's encoder once, repacked on the device
    w = O.synth_normal(1 + rank, n_in * n_out, std=0.02)
    raw = torch.from_numpy(O.quantize_weights(14, w, n_in, n_out)).to(dev)
    packed = torch.empty(GEMV_COPIES, wb, dtype=torch.uint8, device=dev)
    for i in range(GEMV_COPIES):
        ops.pack_weights(14, raw, packed[i], n_in, n_out, stream)
    del raw
    x_host = torch.from_numpy(O.synth_normal(2 + rank, n_in * nc)).pin_memory()
    x_dev = x_host.to(dev)
    xq = torch.empty(ops.native_q8_1_bytes(n_in, nc), dtype=torch.uint8, device=dev)
    y = torch.empty(nc * n_out, dtype=torch.float32, device=dev)
    y_host = torch.empty(nc * n_out, dtype=torch.float32).pin_memory()
    ops.native_quantize_q8_1(x_dev, xq, n_in, nc, stream)

    def step(i):
        ops.mmvq_packed(14, packed[i % GEMV_COPIES], xq, y, n_in, n_out, nc, stream)

    for i in range(args.warmup):
        step(i)
    barrier(pg, dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        for i in range(args.steps):
            step(i)
        ev1.record(stream)
        barrier(pg, dev)
    t_ms = ev0.elapsed_time(ev1)
    t_ms = max_over_ranks(t_ms, pg, dev)
    status = ops.device_status()

    # e2e through the public API with host buffers: H2D x (pinned), quantize, GEMV, D2H y
    def e2e_step(i):
        x_dev.copy_(x_host, non_blocking=True)
        ops.native_quantize_q8_1(x_dev, xq, n_in, nc, stream)
        ops.mmvq_packed(14, packed[i % GEMV_COPIES], xq, y, n_in, n_out, nc, stream)
        y_host.copy_(y, non_blocking=True)

    for i in range(args.warmup):
        e2e_step(i)
    barrier(pg, dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        e2e_step(i)
    e1.record(stream)
    barrier(pg, dev)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), pg, dev)

    algo = gemv_algorithmic_bytes(n_in, n_out, nc)
    per_launch_s = t_ms / 1e3 / args.steps
    achieved = algo / per_launch_s / 1e9
    peak, peak_kind = measured_peaks()
    value = algo * args.steps * world / (t_ms / 1e3) / 1e9
    line = {
        "metric": "Q6_K x Q8_1 GEMV HBM GB/s (12288x4096, ncols 2)",
        "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(t_ms / args.steps, 5), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "q6_k x q8_1 int8 dp4a, fp32 accumulate", "data": "synthetic",
        "config": {"workload": "config1-gemv", "n_in": n_in, "n_out": n_out, "ncols": nc,
                   "weights": "Q6_K packed tiles, 8 rotating copies (330 MB) > L2 126 MB",
                   "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": None, "peak_source": peak_kind,
                     "algorithmic_bytes_per_launch": algo},
        "e2e": {"value": round(algo * args.steps * world / (e2e_ms / 1e3) / 1e9, 1), "unit": "GB/s",
                "h2d_bytes_per_step": n_in * nc * 4, "d2h_bytes_per_step": n_out * nc * 4},
        "gpu_launches": args.steps,
        "device_status": status,
        "clocks": clk.summary(),
    }
    return line


def cpu_baseline_gemv(sample_rows=4096):
    """The oracle (C, OpenMP over the host cores) on a bounded sample of config 1: sample_rows x 4096."""
    from oracle import oracle as O

    n_in, nc = GEMV_N_IN, GEMV_NCOLS
    w = O.synth_normal(1, n_in * sample_rows, std=0.02)
    raw = O.quantize_weights(14, w, n_in, sample_rows)
    xq = O.quantize_q8_1(O.synth_normal(2, n_in * nc), n_in, nc)
    O.mmvq(14, raw, xq, n_in, sample_rows, nc)
    reps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < 10.0 or reps < 2:
        O.mmvq(14, raw, xq, n_in, sample_rows, nc)
        reps += 1
    dt = (time.perf_counter() - t0) / reps
    algo = gemv_algorithmic_bytes(n_in, sample_rows, nc)
    return {"value": round(algo / dt / 1e9, 3), "unit": "GB/s", "cores": O.num_threads(), "kind": "port",
            "sample": f"{sample_rows}x{n_in} rows of config 1, ncols {nc}, {reps} reps"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="rapier", choices=["rapier", "reference"])
    ap.add_argument("--workload", default="gemv", choices=["gemv"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
        base = cpu_baseline_gemv()
        line = {"impl": "reference", "metric": "Q6_K x Q8_1 GEMV HBM GB/s (12288x4096, ncols 2)",
                "value": base["value"], "unit": base["unit"], "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "q6_k x q8_1 int8, fp32 accumulate", "data": "synthetic",
                "config": {"workload": "config1-gemv", "n_in": GEMV_N_IN, "n_out": GEMV_N_OUT,
                           "ncols": GEMV_NCOLS},
                "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": base["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    rank, world, local, pg = dist_init(args.gpus)
    line = run_gemv(args, rank, world, local, pg)
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_gemv()
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
