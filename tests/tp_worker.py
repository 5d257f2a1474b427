"""One rank of the tensor-parallel decode check (launched by tests/test_tp_gpu.py through
torch.distributed.run, one process per GPU). Rank 0 writes the results to the JSON path in argv[1].

The model is a 4-layer, 2048-wide geometry (the smallest whose row-parallel inputs split over 2 ranks
into whole 1024-value tiles). Every rank: teacher-forced steps (its logits shard and the global argmax),
then greedy and MTP generations. Rank 0 also runs the same steps on a single-GPU engine for reference."""
import json
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from rapier_b200.engine import Engine, config_9b  # noqa: E402


def mid_config(max_ctx=512, seed=3):
    c = config_9b(max_ctx, seed)
    c.n_layer, c.n_embd, c.n_ff, c.n_vocab = 4, 2048, 4096, 4096
    c.ssm_h_k, c.ssm_h_v, c.n_head, c.n_head_kv = 8, 16, 8, 2
    return c


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    cfg = mid_config()
    eng = Engine(cfg, device=rank, tp_rank=rank, tp_size=world)
    eng.connect_tp()
    dist.barrier()
    toks = [int(t) for t in np.random.default_rng(5).integers(0, cfg.n_vocab, 24)]
    eng.reset()
    shards, ams = [], []
    for pos, t in enumerate(toks):
        lg, am = eng.step([t], pos)
        shards.append(lg[0].tolist())
        ams.append(am[0])
    prompt = [int(t) for t in np.random.default_rng(6).integers(0, cfg.n_vocab, 16)]
    g0, _ = eng.generate(prompt, 96, mtp=False)
    g1, st = eng.generate(prompt, 96, mtp=True)
    mine = {"rank": rank, "shards": shards, "argmax": ams, "greedy": g0.tolist(), "mtp": g1.tolist(),
            "mtp_steps": st["mtp_steps"]}
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
