"""Host-side logic of tensor-parallel decode, on the CPU: the rank layout bench.py uses, and the exchange of
the ranks' peer-memory handles over torch.distributed (gloo, world size 2) that Engine.connect_tp does
before rk_engine_tp_connect (a stand-in engine records what it is handed)."""
import os
import socket

import torch.multiprocessing as mp


def test_tp_layout():
    import bench

    assert bench.tp_layout(1) == (1, 1)
    assert bench.tp_layout(2) == (2, 1)
    assert bench.tp_layout(4) == (4, 1)
    assert bench.tp_layout(8) == (8, 1)
    assert bench.tp_layout(6) == (2, 3)
    assert bench.tp_layout(3) == (1, 3)


class _StandIn:
    """Engine.connect_tp's view of an engine: tp_rank / tp_size, tp_export, tp_connect."""

    def __init__(self, rank, n):
        self.tp_rank, self.tp_size = rank, n
        self.got = None

    def tp_export(self):
        return bytes([self.tp_rank + 1]) * 64

    def tp_connect(self, handles):
        self.got = handles


def _worker(rank, world, port, q):
    import torch.distributed as dist

    from rapier_b200.engine import Engine

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    eng = _StandIn(rank, world)
    Engine.connect_tp(eng)  # the unbound method on the stand-in: the exchange code under test
    q.put((rank, [h[0] for h in eng.got], [len(h) for h in eng.got]))
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_connect_tp_exchanges_handles_in_rank_order():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        rank, firsts, lens = q.get(timeout=120)
        got[rank] = (firsts, lens)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in range(2):
        assert got[rank] == ([1, 2], [64, 64])
