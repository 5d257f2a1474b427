"""The serving session and the --serve protocol (the reference's serve loop, src/qwythos.cpp:2593-2812) on
the tiny synthetic model: a session run generates what rk_engine_generate generates; runs continue the
context (every emitted token but a final end-of-sequence id is ingested); MTP and plain greedy give the same
ids through the session; generation stops after the end-of-sequence id; the rapier_serve binary answers the
protocol's lines with the session's ids and top-k lists."""
import json
import os
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def eng():
    from rapier_b200.engine import Engine, config_tiny

    e = Engine(config_tiny(max_ctx=256))
    yield e
    e.close()


P1 = [11, 22, 33, 44, 55, 66, 77]
P2 = [5, 6, 7]


@pytest.mark.parametrize("mtp", [False, True])
def test_run_equals_generate(eng, mtp):
    want, _ = eng.generate(P1, 24, mtp=False)
    eng.session_reset()
    got, st, lg = eng.session_run(P1, 24, mtp=mtp, first_logits=True)
    assert list(got) == list(want)
    assert int(np.argmax(lg)) == int(got[0])
    assert eng.session_pos == len(P1) + 24  # the last emitted token counts (pending)


@pytest.mark.parametrize("mtp", [False, True])
def test_continuation(eng, mtp):
    eng.session_reset()
    out1, _, _ = eng.session_run(P1, 9, mtp=mtp)
    out2, _, _ = eng.session_run(P2, 12, mtp=mtp)
    ctx = P1 + list(out1) + P2
    want, _ = eng.generate(ctx, 12, mtp=False)
    assert list(out2) == list(want)
    assert eng.session_pos == len(ctx) + 12


def test_pending_only_run(eng):
    eng.session_reset()
    a, _, _ = eng.session_run(P1, 5)
    b, _, _ = eng.session_run([], 5)  # ingests the pending token only
    want, _ = eng.generate(P1, 10)
    assert list(a) + list(b) == list(want)


@pytest.mark.parametrize("mtp", [False, True])
@pytest.mark.parametrize("k", [0, 2, 5])
def test_stops_after_eos(eng, mtp, k):
    ref, _ = eng.generate(P1, 16)
    eos = int(ref[k])
    first = list(ref).index(eos)  # the first occurrence ends the run
    eng.session_reset()
    out, _, _ = eng.session_run(P1, 16, mtp=mtp, eos=eos)
    assert list(out) == list(ref[:first + 1])
    # the end-of-sequence id is not part of the context: the next run continues after ref[:first]
    out2, _, _ = eng.session_run(P2, 8, mtp=mtp)
    want, _ = eng.generate(P1 + list(ref[:first]) + P2, 8)
    assert list(out2) == list(want)


def test_context_full(eng):
    from rapier_b200 import _lib

    eng.session_reset()
    with pytest.raises(_lib.RkError) as ei:
        eng.session_run(list(range(1, 200)), 100)
    assert ei.value.code == _lib.RK_ERANGE
    eng.session_reset()


def _serve(lines, *extra):
    exe = os.path.join(ROOT, "rapier_b200", "rapier_serve")
    r = subprocess.run([exe, "--synthetic", "tiny", "--seed", "7", "--max-ctx", "256", "--serve", *extra],
                       input="".join(json.dumps(x, separators=(",", ":")) + "\n" for x in lines),
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    return [json.loads(x) for x in r.stdout.splitlines() if x.strip()]


def test_serve_protocol(eng):
    out = _serve([{"op": "reset"},
                  {"op": "run", "tokens": P1, "gen": 10, "mtp": True},
                  {"op": "run", "tokens": P2, "gen": 6, "mtp": False, "topk": 5},
                  {"op": "run", "tokens": [], "gen": 3},
                  {"op": "reset"},
                  {"op": "run", "tokens": list(range(1, 250)), "gen": 20}])
    assert out[0] == {"ok": True, "op": "reset"}
    ids1 = [d["id"] for d in out[1:11]]
    assert out[11] == {"done": True, "pos": len(P1) + 10}
    assert len(out[1]["top"]) == 40 and all(d["top"] == [] for d in out[2:11])
    assert out[1]["top"][0][0] == ids1[0]
    ids2 = [d["id"] for d in out[12:18]]
    for d in out[12:18]:
        top = d["top"]
        assert len(top) == 5 and top[0][0] == d["id"]
        assert all(top[i][1] >= top[i + 1][1] for i in range(4))
    assert out[18] == {"done": True, "pos": len(P1) + 10 + len(P2) + 6}
    assert out[19] == {"error": "need tokens and gen"}
    assert out[20] == {"ok": True, "op": "reset"}
    assert out[21] == {"error": "context full; send op reset"}
    # the same ids through the Python session
    eng.session_reset()
    a, _, _ = eng.session_run(P1, 10, mtp=True)
    b, _, _ = eng.session_run(P2, 6)
    assert ids1 == list(a) and ids2 == list(b)


def test_cli_generation(eng):
    exe = os.path.join(ROOT, "rapier_b200", "rapier_serve")
    r = subprocess.run([exe, "--synthetic", "tiny", "--seed", "7", "--max-ctx", "256", "--prompt",
                        ",".join(map(str, P1)), "--gen", "12", "--mtp"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    d = json.loads(r.stdout.strip().splitlines()[-1])
    want, _ = eng.generate(P1, 12)
    assert d["ids"] == list(want)
