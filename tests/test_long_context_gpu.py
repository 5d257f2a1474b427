"""Decode after a long synthetic context (rk_engine_session_fill: seeded fp16 K/V and GDN states): chunks of
512 tokens scored in two 256-token passes each, the MTP stream equal to the greedy stream, and the two
executors bit for bit, at a 20000-token context."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FILL = 20000
P = [9, 99, 999, 3, 33]


@pytest.fixture(scope="module")
def pair():
    from rapier_b200.engine import Engine, config_tiny

    cfg = config_tiny(max_ctx=FILL + 256)
    g, p = Engine(cfg, mode="graph"), Engine(cfg, mode="persistent")
    yield g, p
    p.close()
    g.close()


def test_mtp_equals_greedy_after_fill(pair):
    g, _ = pair
    g.session_fill(FILL, 3)
    a, _, _ = g.session_run(P, 40, mtp=False)
    g.session_fill(FILL, 3)
    b, st, _ = g.session_run(P, 40, mtp=True)
    assert list(a) == list(b) and st["mtp_steps"] > 0
    assert g.session_pos == FILL + len(P) + 40


def test_executors_agree_after_fill(pair):
    g, p = pair
    outs = []
    for e in (g, p):
        e.session_fill(FILL, 5)
        ids, _, lg = e.session_run(P, 12, mtp=True, first_logits=True)
        outs.append((list(ids), lg.view(np.uint32).copy()))
    assert outs[0][0] == outs[1][0]
    assert np.array_equal(outs[0][1], outs[1][1])


def test_fill_is_deterministic_and_seeded(pair):
    g, _ = pair
    g.session_fill(FILL, 11)
    a, _, la = g.session_run(P, 1, first_logits=True)
    g.session_fill(FILL, 11)
    b, _, lb = g.session_run(P, 1, first_logits=True)
    g.session_fill(FILL, 12)
    _, _, lc = g.session_run(P, 1, first_logits=True)
    assert np.array_equal(la, lb) and not np.array_equal(la, lc)
