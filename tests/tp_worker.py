"""One rank of the tensor-parallel decode checks (launched by tests/test_tp_gpu.py through
torch.distributed.run, one process per GPU). Rank 0 writes the results to the JSON path in argv[1].

argv[2] = "check" (default): teacher-forced steps (every rank's logits shard and the global argmax), then
greedy and MTP generations; rank 0 also runs the same steps on a single-GPU engine for reference.
argv[2] = "fail": after a reference generation, rank 0 runs one step that rank 1 skips, so rank 0's
cross-rank waits give up (RK_TP_WAIT_MS, set short by the launcher); then every rank resyncs and resets
and the generation is repeated. The host barriers are gloo's; no rank leaves a kernel in flight.

argv[2] = "exec": the same teacher-forced steps and generations on the persistent executor and on the graph
executor (one kernel per op; the exchange inside the GEMV and argmax kernels); rank 0 writes both.

argv[3] = geometry: "mid" (2048 wide, 4 layers: splits over 2 ranks into whole tiles), "tiny" (1024 wide, 4
q heads and 1 kv head: over 2 ranks each keeps the shared kv head and pads its 512-value row-parallel
inputs to a tile, the 8-rank layout of the 9B geometry on 2 GPUs) or "9b4" (the 9B geometry cut to 4
layers and a 32768-token vocabulary: splits over 2, 4 and 8 ranks, with replicated kv heads at 8)."""
import json
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from rapier_b200 import ops  # noqa: E402
from rapier_b200._lib import RK_ECUDA, RkError  # noqa: E402
from rapier_b200.engine import Engine, config_9b  # noqa: E402


def geometry(name, max_ctx=512, seed=3):
    c = config_9b(max_ctx, seed)
    if name == "mid":
        c.n_layer, c.n_embd, c.n_ff, c.n_vocab = 4, 2048, 4096, 4096
        c.ssm_h_k, c.ssm_h_v, c.n_head, c.n_head_kv = 8, 16, 8, 2
    elif name == "tiny":
        c.n_layer, c.n_embd, c.n_ff, c.n_vocab = 4, 1024, 2048, 4096
        c.ssm_h_k, c.ssm_h_v, c.n_head, c.n_head_kv = 4, 8, 4, 1
    else:
        c.n_layer, c.n_vocab = 4, 32768
    return c


def run_executors(cfg, rank, world):
    toks = [int(t) for t in np.random.default_rng(5).integers(0, cfg.n_vocab, 16)]
    prompt = [int(t) for t in np.random.default_rng(6).integers(0, cfg.n_vocab, 16)]
    mine = {"rank": rank}
    for ex in ("persistent", "graph"):
        eng = Engine(cfg, device=rank, mode=ex, tp_rank=rank, tp_size=world)
        eng.connect_tp()
        dist.barrier()
        eng.reset()
        bits, ams = [], []
        for pos, t in enumerate(toks):
            lg, am = eng.step([t], pos)
            bits.append(np.ascontiguousarray(lg[0], np.float32).view(np.uint32).tolist())
            ams.append(am[0])
        g0, _ = eng.generate(prompt, 48, mtp=False)
        g1, st = eng.generate(prompt, 48, mtp=True)
        mine[ex] = {"mode": eng.mode, "bits": bits, "argmax": ams, "greedy": g0.tolist(), "mtp": g1.tolist(),
                    "mtp_steps": st["mtp_steps"], "status": ops.device_status()}
        dist.barrier()
        eng.close()
        dist.barrier()
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    if rank == 0:
        with open(sys.argv[1], "w") as f:
            json.dump({"ranks": gathered}, f)
    dist.barrier()
    dist.destroy_process_group()


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    mode = sys.argv[2] if len(sys.argv) > 2 else "check"
    geo = sys.argv[3] if len(sys.argv) > 3 else "mid"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    cfg = geometry(geo)
    if mode == "exec":
        run_executors(cfg, rank, world)
        return
    eng = Engine(cfg, device=rank, tp_rank=rank, tp_size=world)
    eng.connect_tp()
    dist.barrier()
    prompt = [int(t) for t in np.random.default_rng(6).integers(0, cfg.n_vocab, 16)]
    if mode == "fail":
        g0, _ = eng.generate(prompt, 24, mtp=False)
        dist.barrier()
        err, status = None, 0
        if rank == 0:  # rank 1 skips this step: rank 0's waits for its partial sums give up
            try:
                eng.step([5], 0, want_logits=False)
            except RkError as e:
                err = e.code
            status = ops.device_status()
        dist.barrier()
        eng.tp_resync()
        dist.barrier()
        eng.reset()
        g1, _ = eng.generate(prompt, 24, mtp=False)
        g2, st = eng.generate(prompt, 24, mtp=True)
        mine = {"rank": rank, "err": err, "status": status, "before": g0.tolist(), "after": g1.tolist(),
                "after_mtp": g2.tolist(), "final_status": ops.device_status()}
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        eng.close()
        if rank == 0:
            with open(sys.argv[1], "w") as f:
                json.dump({"ranks": gathered, "ecuda": RK_ECUDA}, f)
        dist.barrier()
        dist.destroy_process_group()
        return
    toks = [int(t) for t in np.random.default_rng(5).integers(0, cfg.n_vocab, 24)]
    eng.reset()
    shards, ams = [], []
    for pos, t in enumerate(toks):
        lg, am = eng.step([t], pos)
        shards.append(lg[0].tolist())
        ams.append(am[0])
    g0, _ = eng.generate(prompt, 96, mtp=False)
    g1, st = eng.generate(prompt, 96, mtp=True)
    mine = {"rank": rank, "shards": shards, "argmax": ams, "greedy": g0.tolist(), "mtp": g1.tolist(),
            "mtp_steps": st["mtp_steps"], "status": ops.device_status()}
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    eng.close()
    if rank == 0:
        ref = Engine(cfg, device=0)
        ref.reset()
        ref_logits, ref_am = [], []
        for pos, t in enumerate(toks):
            lg, am = ref.step([t], pos)
            ref_logits.append(lg[0].tolist())
            ref_am.append(am[0])
        r0, _ = ref.generate(prompt, 96, mtp=False)
        ref.close()
        with open(sys.argv[1], "w") as f:
            json.dump({"ranks": gathered, "ref_logits": ref_logits, "ref_argmax": ref_am, "ref_greedy": r0.tolist()}, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
