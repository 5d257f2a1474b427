"""Batched prompt ingest (the reference's serve ingest, src/qwythos.cpp:2151-2502): 4-column trunk passes
without the lm_head, each column bitwise the single-token pass. The logits after ingesting a prompt this way
equal, bit for bit, those after stepping its tokens one at a time, in both executors; generation and
sessions over chunked prompts give the per-token ids."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", params=["persistent", "graph"])
def eng(request):
    from rapier_b200.engine import Engine, config_tiny

    e = Engine(config_tiny(max_ctx=256), mode=request.param)
    yield e
    e.close()


def _stepped_logits(eng, toks):
    eng.reset()
    lg = None
    for pos, t in enumerate(toks):
        lg, _ = eng.step([t], pos)
    return lg[0]


@pytest.mark.parametrize("n", [5, 8, 13, 18])
def test_chunked_ingest_bitwise(eng, n):
    toks = [int(t) for t in np.random.default_rng(n).integers(0, 4096, n)]
    want = _stepped_logits(eng, toks)
    eng.session_reset()
    ids, _, lg = eng.session_run(toks, 1, first_logits=True)
    assert np.array_equal(lg.view(np.uint32), want.view(np.uint32))
    assert ids[0] == int(np.argmax(want))


def test_generate_after_chunked_prompt(eng):
    toks = [int(t) for t in np.random.default_rng(3).integers(0, 4096, 21)]
    ids, _ = eng.generate(toks, 10, mtp=False)
    eng.reset()
    seq = list(toks)
    for pos in range(len(toks) + 9):
        _, am = eng.step([seq[pos]], pos, want_logits=False)
        if pos >= len(toks) - 1:
            assert am[0] == ids[pos - len(toks) + 1]
            seq.append(am[0])
    ids_mtp, _ = eng.generate(toks, 10, mtp=True)
    assert list(ids_mtp) == list(ids)


def test_session_continuation_chunked(eng):
    p1 = list(range(100, 111))
    p2 = list(range(300, 309))
    eng.session_reset()
    a, _, _ = eng.session_run(p1, 6)
    b, _, _ = eng.session_run(p2, 6)  # the pending token and 9 new ones: two 4-column passes, then singles
    want, _ = eng.generate(p1 + list(a) + p2, 6)
    assert list(b) == list(want)
