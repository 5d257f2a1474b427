"""Decode after a long synthetic context (rk_engine_session_fill: seeded fp16 K/V and GDN states) in an engine
of 20256 positions (flash-decode chunks of 64 tokens): the MTP stream equal to the greedy stream, the two
executors bit for bit, and a 2-column step bitwise equal to two single-token steps at position 16383, where
a chunk length chosen from the position (32 tokens below 16384, 64 above) would have split the two columns'
keys differently."""
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


def test_two_columns_equal_singles_at_former_chunk_boundary(pair):
    g, _ = pair
    pos = 16383
    g.session_fill(pos, 4)
    lg2, _ = g.step([7, 8], pos)
    g.session_fill(pos, 4)
    s0, _ = g.step([7], pos)
    s1, _ = g.step([8], pos + 1)
    assert np.array_equal(lg2[0].view(np.uint32), s0[0].view(np.uint32))
    assert np.array_equal(lg2[1].view(np.uint32), s1[0].view(np.uint32))


def test_mtp_equals_greedy_across_former_chunk_boundary(pair):
    g, _ = pair
    g.session_fill(16370, 6)
    a, _, _ = g.session_run(P, 40, mtp=False)
    g.session_fill(16370, 6)
    b, st, _ = g.session_run(P, 40, mtp=True)
    assert list(a) == list(b) and st["mtp_steps"] > 0
