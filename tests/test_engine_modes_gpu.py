"""The engine's two executors against each other: the persistent decode kernel (one cooperative launch per
step program, weight rings streaming across ops, grid barriers between ops) and the graph of one kernel
per op. They run the same op bodies and the same GEMV arithmetic, so logits, argmax ids and token streams
must be bitwise equal: teacher-forced 1- and 2-column steps, steps that cross flash-decode chunk
boundaries, and greedy / MTP generations (the persistent kernel loops over a whole generation in one
launch)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pair(cuda):
    from rapier_b200.engine import Engine, config_tiny

    cfg = config_tiny(max_ctx=768, seed=5)
    g, p = Engine(cfg, mode="graph"), Engine(cfg, mode="persistent")
    assert g.mode == "graph" and p.mode == "persistent"
    yield g, p
    g.close()
    p.close()


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def test_teacher_forced_steps_bitwise(pair):
    g, p = pair
    g.reset()
    p.reset()
    toks = np.random.default_rng(3).integers(0, 4096, 24)
    pos = 0
    for i, t in enumerate(toks):
        if i % 3 == 2:  # a 2-column pass now and then (the verify width)
            cols = [int(t), int(toks[i - 1])]
        else:
            cols = [int(t)]
        lg, ag = g.step(cols, pos)
        lp, ap = p.step(cols, pos)
        assert np.array_equal(_bits(lg), _bits(lp)), pos
        assert ag == ap
        pos += len(cols)


def test_chunk_boundaries_bitwise(pair):
    """Positions 250..262 and 508..516 in 2-column steps: a step whose two columns straddle the 256-token
    chunk edge (255 | 256) has its new keys owned by two different chunk items."""
    g, p = pair
    g.reset()
    p.reset()
    rng = np.random.default_rng(9)
    pos = 0
    while pos < 520:
        two = (250 <= pos < 262) or (508 <= pos < 516)
        cols = [int(x) for x in rng.integers(0, 4096, 2 if two else 1)]
        want_logits = two or pos % 64 == 0
        lg, ag = g.step(cols, pos, want_logits=want_logits)
        lp, ap = p.step(cols, pos, want_logits=want_logits)
        assert ag == ap, pos
        if want_logits:
            assert np.array_equal(_bits(lg), _bits(lp)), pos
        pos += len(cols)


@pytest.mark.parametrize("mtp", [False, True])
def test_generation_bitwise(pair, mtp):
    g, p = pair
    prompt = list(range(40, 72))
    ig, sg = g.generate(prompt, 150, mtp=mtp)
    ip, sp = p.generate(prompt, 150, mtp=mtp)
    assert np.array_equal(ig, ip)
    assert sp["kernels_per_single_step"] == 1
    if mtp:
        assert sp["mtp_steps"] == sg["mtp_steps"] > 0
        assert sp["mtp_accepted"] == sg["mtp_accepted"]
        assert sp["kernels_per_round"] == 1
    else:
        # 31 prompt positions: seven 4-column prefill passes and three single ones; one launch generates
        assert sp["graph_launches"] == 7 + 3 + 1


def test_mtp_equals_greedy_persistent(pair):
    _, p = pair
    prompt = [7, 1, 4095, 12, 300]
    i0, _ = p.generate(prompt, 200, mtp=False)
    i1, st = p.generate(prompt, 200, mtp=True)
    assert np.array_equal(i0, i1)
    assert st["mtp_steps"] > 0


def test_probe_runs_in_both_modes(pair):
    for e in pair:
        r = e.probe_gemv(ncols=2, iters=2)
        assert r["ms"] > 0 and r["launches"] == 4 * e.cfg.n_layer + 1
