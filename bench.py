"""Benchmark of the rapier_b200 decode hot path (driver contract: one JSON line from rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl rapier|reference] [--workload gemv|decode]

Workloads (synthetic seeded data, no model file):
  decode  config 5 (default): the 9B-shaped qwen35 hybrid (24 GDN + 8 GQA layers, MTP block), random-init
          weights quantized to Q6_K, greedy decode of 400 tokens from a seeded 32-token prompt with exact
          MTP (--no-mtp: config 4). A step is one 400-token generation; tok/s = generated tokens / device
          time of the generation (prefill excluded, as the reference's tok_s, src/qwythos.cpp:3243-3247).
          Weights (6.5 GB) exceed L2, so every token streams them from HBM.
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
# DRAM bytes of one config-1 launch (12288 x 4096, 2 columns) from an ncu capture of this kernel: 41,328,384
# read + 9,216 written, equal to the algorithmic bytes (no re-reads).
GEMV_CONFIG1_NCU_TRAFFIC = 41_337_600


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
                     "frac": round(achieved / peak, 4), "traffic": GEMV_CONFIG1_NCU_TRAFFIC if nc == 2 else None,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch "
                                       "(profiles/mmvq_packed_config1_gemv.md)" if nc == 2 else None,
                     "peak_source": peak_kind, "algorithmic_bytes_per_launch": algo},
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


# ------------------------------------------------------------------------------------------------------
# decode workload (configs 4 / 5)
# ------------------------------------------------------------------------------------------------------
N_PROMPT, N_GEN = 32, 400
# DRAM bytes per GEMV launch of one 2-column (verify) trunk step, 32 layers + lm_head, from an ncu capture of
# the 4-layer 2-column pass (profiles/mmvq_packed_decode_2col_pass.md): 24 x GDN layer + 8 x attention layer
# + lm_head, / 129 launches (the engine's 2-column launches: 16 warps per CTA, paired where that helps).
DECODE_2COL_NCU_TRAFFIC = 50_690_401


def tp_layout(world: int) -> tuple:
    """(tensor-parallel size, groups) for `world` GPUs: one tensor-parallel group of 1, 2, 4 or 8 ranks (the
    9B geometry's head and row-parallel splits), else groups of 4 or 2 (independent streams)."""
    if world in (1, 2, 4, 8):
        return world, 1
    for tp in (4, 2):
        if world % tp == 0:
            return tp, world // tp
    return 1, world


def decode_config(args, world: int) -> dict:
    """The decode line's `config`, from the arguments only (the same dict on both arms)."""
    tp, groups = tp_layout(world)
    fill, mtp = args.ctx_fill, not args.no_mtp
    par = "single GPU" if world == 1 else (f"tensor parallel x{tp}" + (f", {groups} independent groups" if groups > 1 else ""))
    return {"workload": "config5-decode-mtp" if mtp else "config4-decode", "model": "qwen35-9b-shaped",
            "layers": "24 GDN + 8 GQA (+1 MTP block)", "n_prompt": N_PROMPT, "n_gen": args.gen,
            "ctx": (fill + N_PROMPT + args.gen) if fill else args.ctx,
            "kv_context": fill + N_PROMPT if fill else N_PROMPT, "parallelism": par, "tensor_parallel": tp,
            "groups": groups, "l2": "6.5 GB of weights per token > 126 MB L2"}


def run_decode(args, rank, world, local, pg):
    import torch

    from rapier_b200.engine import Engine, config_9b

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    tp, groups = tp_layout(world)
    grp, tp_rank = rank // tp, rank % tp
    group = None
    if tp > 1:
        subgroups = [pg.new_group(list(range(g * tp, (g + 1) * tp))) for g in range(groups)]
        group = subgroups[grp]
    fill = args.ctx_fill
    cfg = config_9b(max_ctx=max(args.ctx, fill + N_PROMPT + args.gen + 64) if fill else args.ctx, seed=1 + grp)
    eng = Engine(cfg, device=local, tp_rank=tp_rank, tp_size=tp)
    if tp > 1:
        eng.connect_tp(group)
        barrier(pg, dev)
    prompt = [int(t) for t in np.random.default_rng(1234 + grp).integers(0, cfg.n_vocab, N_PROMPT)]
    mtp = not args.no_mtp
    n_gen = args.gen

    def one_generation():
        if fill:  # decode after a synthetic context of `fill` tokens (seeded caches, rk_engine_session_fill)
            eng.session_fill(fill, 7 + grp)
            ids, st, _ = eng.session_run(prompt, n_gen, mtp=mtp)
            return ids, st
        return eng.generate(prompt, n_gen, mtp=mtp)

    for _ in range(args.warmup):
        ids0, _ = one_generation()
    barrier(pg, dev)
    gen_ms, stats = 0.0, None
    t0 = time.perf_counter()
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            ids, st = one_generation()
            gen_ms += st["gen_ms"]
            stats = st
        barrier(pg, dev)
    wall_s = time.perf_counter() - t0
    gen_ms = max_over_ranks(gen_ms, pg, dev)
    wall_s = max_over_ranks(wall_s, pg, dev)
    tokens = n_gen * args.steps * groups
    forced = None
    if mtp:
        # the same generations with every draft candidate forced to the token the greedy stream has at its
        # position (rk_engine_force_candidates): acceptance 1.0, the stream unchanged; what exact MTP gives
        # once the draft is right, on this engine
        seq = list(prompt) + [int(t) for t in ids0]
        if fill:
            seq = [-1] * fill + seq
        eng.force_candidates(seq)
        f_ms, f_st = 0.0, None
        for _ in range(args.steps):
            ids_f, st_f = one_generation()
            assert np.array_equal(ids_f, ids0), "forced-candidate stream differs from the greedy stream"
            f_ms += st_f["gen_ms"]
            f_st = st_f
        eng.force_candidates(None)
        f_ms = max_over_ranks(f_ms, pg, dev)
        forced = {"tok_s": round(tokens / (f_ms / 1e3), 2), "ms_per_generation": round(f_ms / args.steps, 3),
                  "rounds": f_st["mtp_steps"], "accepted": f_st["mtp_accepted"],
                  "acceptance": round(f_st["mtp_accepted"] / max(1, f_st["mtp_steps"]), 4),
                  "note": "candidates forced to the greedy stream's tokens (test hook); same tokens emitted"}
    probe = eng.probe_gemv(ncols=2 if mtp else 1, iters=20)
    persistent = eng.mode == "persistent"
    eng.close()
    peak, peak_kind = measured_peaks()
    per_launch_s = probe["ms"] / 1e3 / (probe["iters"] * probe["launches"])
    algo_per_launch = probe["algo_bytes"] / probe["launches"]
    achieved = algo_per_launch / per_launch_s / 1e9
    rounds = stats["mtp_steps"]
    if persistent:  # one kernel per program run (a whole greedy generation is one run)
        launches_per_gen = stats["graph_launches"]
    else:
        launches_per_gen = ((stats["graph_launches"] - rounds) * stats["kernels_per_single_step"] +
                            rounds * stats["kernels_per_round"])
    cfgd = decode_config(args, world)
    line = {
        "metric": "greedy decode tok/s (1 B200, exact MTP)" if mtp else "greedy decode tok/s (1 B200, no MTP)",
        "value": round(tokens / (gen_ms / 1e3), 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(gen_ms / args.steps, 3), "higher_is_better": True,
        "scaling": "strong" if (world > 1 and groups == 1) else "weak", "vs_baseline": None,
        "dtype": "q6_k x q8_1 int8 dp4a, fp32 accumulate, fp16 KV",
        "data": "synthetic (random-init weights, seeded prompt)",
        "config": cfgd,
        "executor": "persistent" if persistent else "graph",
        "mtp": {"rounds": rounds, "accepted": stats["mtp_accepted"],
                "acceptance": round(stats["mtp_accepted"] / rounds, 4) if rounds else None,
                "single_steps": stats["single_steps"], "forced_acceptance_1": forced} if mtp else None,
        "roofline": {"bound": "hbm",
                     "kernel": ("persistent_kernel (the GEMV ops of one trunk step, one launch)" if persistent else
                                "mmvq_packed_kernel (all GEMVs of one trunk step, graph replay)"),
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": DECODE_2COL_NCU_TRAFFIC if (mtp and not persistent and tp == 1) else None,
                     "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of the 4-layer 2-column pass, "
                                        "scaled to 32 layers (profiles/mmvq_packed_decode_2col_pass.md)")
                     if (mtp and not persistent and tp == 1) else None,
                     "peak_source": peak_kind, "algorithmic_bytes_per_launch": round(algo_per_launch),
                     "gemv_ops": probe["launches"], "avg_gemv_us": round(per_launch_s * 1e6, 3),
                     "per_gpu": tp > 1},
        "e2e": {"value": round(tokens / wall_s, 2), "unit": "tok/s",
                "h2d_bytes_per_step": N_PROMPT * 4 + 32 * (N_PROMPT + 2),
                "d2h_bytes_per_step": n_gen * 4 + 4 * rounds + 96},
        "gpu_launches": launches_per_gen * args.steps,
        "clocks": clk.summary(),
    }
    return line


def run_pass(args):
    """Four passes (--cols 1: single tokens; 2: the verify's two columns) of a 9B-shaped model cut to
    --layers layers (the full lm_head): the small case for an ncu capture of the step kernels (the kernels the
    32-layer engine runs); with --ctx-fill N the passes run after a synthetic context of N tokens. Not a
    bench line: prints the four pass times."""
    import torch

    from rapier_b200.engine import Engine, config_9b

    torch.cuda.set_device(0)
    fill = args.ctx_fill
    cfg = config_9b(max_ctx=max(args.ctx, fill + 64) if fill else args.ctx, seed=1)
    cfg.n_layer = args.layers
    eng = Engine(cfg)
    if fill:
        eng.session_fill(fill, 7)
    times = []
    toks = [5, 17, 99, 1000, 7, 250, 31, 4096]
    for i in range(4):
        t0 = time.perf_counter()
        eng.step(toks[args.cols * i:args.cols * (i + 1)], fill + args.cols * i, want_logits=False)
        times.append(round((time.perf_counter() - t0) * 1e3, 3))
    print(json.dumps({"workload": "pass", "layers": args.layers, "cols": args.cols, "step_ms_wall": times}), flush=True)
    eng.close()


def cpu_baseline_decode(budget_s=20.0, mtp=True):
    """The oracle (C restatement, OpenMP over the host cores) on one GDN layer, one attention layer, the MTP
    block and the lm_head of the 9B shape; a token's time is extrapolated as 24 x GDN + 8 x attention +
    head. With exact MTP at this model's acceptance of 0 (random weights), every round emits one token and
    costs two trunk columns and two draft columns; the oracle runs columns one after the other."""
    from oracle import oracle as O
    from oracle.model import Model, config_9b

    cfg = config_9b(max_ctx=64, seed=1, n_layer=4)  # layers 0..2 GDN, 3 attention; layers 0 and 3 are timed
    t_gen = time.perf_counter()
    m = Model(cfg, only_layers=(0, 3), with_embed=False, with_draft=mtp)
    t_gen = time.perf_counter() - t_gen
    H = cfg.n_embd
    x = O.synth_normal(3, H)
    xp = O.row_sumsq_partials(x)
    timings = {"gdn": [], "attn": [], "head": [], "draft": []}
    t_end = time.perf_counter() + budget_s
    pos = 0
    while (time.perf_counter() < t_end or pos < 2) and pos < cfg.max_ctx:
        for kind, il in (("gdn", 0), ("attn", 3)):
            t0 = time.perf_counter()
            m.layer(il, x, xp, pos)
            timings[kind].append(time.perf_counter() - t0)
        t0 = time.perf_counter()
        m.head(x, xp)
        timings["head"].append(time.perf_counter() - t0)
        if mtp:  # the draft without its embedding row: eh_proj, the nextn layer, the head
            t0 = time.perf_counter()
            ehq = O.quantize_q8_1(np.concatenate([x, x]), 2 * H, 1)
            dx = O.mmvq(O.TYPE_Q6_K, m.eh_proj, ehq, 2 * H, H)
            dx, dxp = m._attention(m.draft_layer, m.draft_kv, dx, O.row_sumsq_partials(dx), pos)
            dx, dxp = m._ffn(m.draft_layer, dx, dxp)
            O.mmvq(O.TYPE_Q6_K, m.lm_head, O.rms_quant_q8_1(dx, m.shnorm, dxp, m.eps), H, cfg.n_vocab)
            timings["draft"].append(time.perf_counter() - t0)
        pos += 1
    med = {k: statistics.median(v) for k, v in timings.items() if v}
    t_tok = 24 * med["gdn"] + 8 * med["attn"] + med["head"]
    if mtp:
        t_out = 2 * (t_tok + med["draft"])
        how = (f"exact MTP at acceptance 0: a round = 2 trunk columns + 2 draft columns = "
               f"2 x ({t_tok * 1e3:.1f} + {med['draft'] * 1e3:.1f}) ms per emitted token")
    else:
        t_out = t_tok
        how = f"no MTP: {t_tok * 1e3:.1f} ms per token"
    return {"value": round(1.0 / t_out, 4), "unit": "tok/s", "cores": O.num_threads(), "kind": "port",
            "sample": f"{pos} positions through 1 GDN + 1 attention layer + lm_head (+ the MTP block) of the 9B "
                      f"shape; token time extrapolated as 24 GDN + 8 attention + head; {how} (weights generated "
                      f"in {t_gen:.1f} s, untimed)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", default="rapier", choices=["rapier", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode", "gemv", "pass"],
                    help="pass: four single-token steps of a --layers model (a small case for ncu captures)")
    ap.add_argument("--layers", type=int, default=8, help="pass: decoder layers of the 9B-shaped model")
    ap.add_argument("--cols", type=int, default=1, choices=[1, 2], help="pass: tokens per pass")
    ap.add_argument("--ctx", type=int, default=512, help="decode: KV capacity (512 or 65536)")
    ap.add_argument("--ctx-fill", type=int, default=0,
                    help="decode: start each generation after a synthetic context of this many tokens (65536: "
                         "config 5 at long context; seeded fp16 K/V and GDN states, rk_engine_session_fill)")
    ap.add_argument("--no-mtp", action="store_true", help="decode: plain greedy (config 4)")
    ap.add_argument("--gen", type=int, default=N_GEN, help="decode: tokens per generation (400; fewer for profiling)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 5 if args.workload == "decode" else 200
    if args.warmup is None:
        args.warmup = 3 if args.workload == "decode" else 10
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
        if args.workload == "decode":
            base = cpu_baseline_decode(mtp=not args.no_mtp)
            metric = "greedy decode tok/s (1 B200, exact MTP)" if not args.no_mtp else "greedy decode tok/s (1 B200, no MTP)"
            cfgd = decode_config(args, args.gpus)
        else:
            base = cpu_baseline_gemv()
            metric = "Q6_K x Q8_1 GEMV HBM GB/s (12288x4096, ncols 2)"
            cfgd = {"workload": "config1-gemv", "n_in": GEMV_N_IN, "n_out": GEMV_N_OUT, "ncols": GEMV_NCOLS}
        line = {"impl": "reference", "metric": metric, "value": base["value"], "unit": base["unit"],
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "q6_k x q8_1 int8, fp32 accumulate",
                "data": "synthetic", "config": cfgd, "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": base["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    if args.workload == "pass":
        run_pass(args)
        return
    rank, world, local, pg = dist_init(args.gpus)
    line = (run_decode if args.workload == "decode" else run_gemv)(args, rank, world, local, pg)
    if rank == 0:
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = (cpu_baseline_decode(mtp=not args.no_mtp) if args.workload == "decode"
                                    else cpu_baseline_gemv())
        print(json.dumps(line), flush=True)
    if pg is not None:
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
