"""The decode engine on the GPU against the CPU oracle of the whole model (oracle/model.py):

* synthetic weights bit-identical to the oracle's generator;
* teacher-forced logits BIT-IDENTICAL to the oracle's, one layer and four layers (the kernels and the
  oracle run the same fp32 operation sequence: the same reductions, and exp / log1p / 1/sqrt from one
  exactly specified recipe), and the greedy token stream identical to the oracle's over 120 tokens;
* the MTP draft head (draft_predict, src/qwythos.cpp:1316-1406) bit-identical to the oracle's draft,
  slot-0 seed included;
* 2-column passes bitwise equal to 1-column passes; MTP stream == greedy stream, with the accept branch
  driven by forced candidates (acceptance 1.0, alternating accept / reject, an accept whose second token
  is the end-of-sequence id), on both executors;
* the 9B shape (4 layers: GDN layers 0-2, attention layer 3, the 248320-row lm_head) bit-identical to the
  oracle at 4 positions, and after a synthetic 65536-token context."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bits_equal(a, b) -> bool:
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


def _assert_bits(got, want, what):
    got = np.asarray(got, np.float32).ravel()
    want = np.asarray(want, np.float32).ravel()
    if not _bits_equal(got, want):
        d = np.abs(got.astype(np.float64) - want)
        i = int(np.argmax(d))
        raise AssertionError(f"{what}: {int(np.sum(got != want))}/{got.size} values differ; worst index {i}: "
                             f"got {got[i]!r} want {want[i]!r} (max |diff| / scale "
                             f"{d[i] / max(np.max(np.abs(want)), 1e-30):.3e})")


@pytest.fixture(scope="module")
def tiny(cuda):
    from rapier_b200.engine import Engine, config_tiny

    cfg = config_tiny(max_ctx=256, seed=7)
    eng = Engine(cfg)
    yield eng
    eng.close()


@pytest.fixture(scope="module")
def tiny_oracle(tiny):
    from oracle.model import Model

    return Model(tiny.cfg)


def test_synthetic_weights_match_oracle_generator(tiny, tiny_oracle):
    from oracle import model as M

    m = tiny_oracle
    assert np.array_equal(tiny.read_tensor(M.T_TOK_EMBD), m.tok_embd)
    assert np.array_equal(tiny.read_tensor(M.T_OUTPUT), m.lm_head)
    assert np.array_equal(tiny.read_tensor(M.T_OUT_NORM).view(np.float32), m.out_norm)
    assert np.array_equal(tiny.read_tensor(M.T_EH_PROJ), m.eh_proj)
    L0 = m.layers[0]
    got = tiny.read_tensor(M.layer_tid(0, M.L_GDN_QKV))
    assert np.array_equal(got, L0["in_proj"][:got.size])
    assert np.array_equal(tiny.read_tensor(M.layer_tid(0, M.L_GDN_A)).view(np.float32), L0["ssm_a"])
    v_bytes = m.nkv * 256 * (m.H // 256) * 210  # the last rows of layer 3's q||k||v group
    assert np.array_equal(tiny.read_tensor(M.layer_tid(3, M.L_ATT_V)), m.layers[3]["in_proj"][-v_bytes:])


@pytest.mark.parametrize("kind", ["gdn", "attn"])
def test_single_layer_logits_bitwise_oracle(cuda, kind):
    """A one-layer model (a GDN layer or an attention layer, plus embedding and lm_head): 12 teacher-forced
    positions exercise the conv ring, the delta-rule state and the KV cache; every logit bit-identical."""
    from oracle.model import Model
    from rapier_b200.engine import Engine, config_tiny

    cfg = config_tiny(max_ctx=64, seed=11, n_layer=1)
    cfg.attn_interval = 1 if kind == "attn" else 4
    eng, m = Engine(cfg), Model(cfg)
    eng.reset()
    toks = np.random.default_rng(2).integers(0, cfg.n_vocab, 12)
    for pos, t in enumerate(toks):
        logits, am = eng.step([t], pos)
        _assert_bits(logits[0], m.forward(int(t), pos), f"{kind} layer, position {pos}")
        assert am[0] == int(np.argmax(logits[0]))
    eng.close()


def test_teacher_forced_logits_bitwise_oracle(tiny, tiny_oracle):
    """The 4-layer model over 16 positions: every logit bit-identical to the oracle's."""
    tiny.reset()
    tiny_oracle.reset()
    toks = np.random.default_rng(0).integers(0, tiny.cfg.n_vocab, 16)
    for pos, t in enumerate(toks):
        logits, am = tiny.step([t], pos)
        want = tiny_oracle.forward(int(t), pos)
        _assert_bits(logits[0], want, f"position {pos}")
        assert am[0] == int(np.argmax(want))


def test_greedy_stream_equals_oracle(tiny, tiny_oracle):
    """120 greedy tokens from a 12-token prompt, token for token against the oracle's greedy decoding."""
    prompt = [int(t) for t in np.random.default_rng(5).integers(0, tiny.cfg.n_vocab, 12)]
    ids, _ = tiny.generate(prompt, 120, mtp=False)
    want = tiny_oracle.generate(prompt, 120)
    assert list(ids) == want


def test_draft_bitwise_oracle(tiny, tiny_oracle):
    """The MTP draft against the oracle's draft_predict restatement: the slot-0 seed (h = 0, emb of the
    first token) without a head, then after every teacher-forced trunk pass at position p the draft at
    position p + 1 on (emb(token p + 1), the final-normed hidden of p): 14 positions, logits and argmax
    bit-identical."""
    m = tiny_oracle
    tiny.reset()
    m.reset()
    toks = [int(t) for t in np.random.default_rng(9).integers(0, tiny.cfg.n_vocab, 16)]
    lg, am = tiny.draft_step(toks[0], 0, h_zero=True)
    want = m.draft(toks[0], 0, h=np.zeros(m.H, np.float32), hp=np.zeros(m.H // 4, np.float32))
    _assert_bits(lg, want, "draft slot 0")
    for p in range(14):
        tiny.step([toks[p]], p, want_logits=False)
        m.forward(toks[p], p)
        lg, am = tiny.draft_step(toks[p + 1], p + 1)
        want = m.draft(toks[p + 1], p + 1)
        _assert_bits(lg, want, f"draft at position {p + 1}")
        assert am == int(np.argmax(want))


def test_two_column_pass_bitwise_equals_single(tiny):
    toks = [5, 17, 1023, 9]
    tiny.reset()
    singles = []
    for pos, t in enumerate(toks):
        lg, _ = tiny.step([t], pos)
        singles.append(lg[0].copy())
    tiny.reset()
    pairs = []
    for pos in range(0, len(toks), 2):
        lg, _ = tiny.step(toks[pos:pos + 2], pos)
        pairs.extend([lg[0].copy(), lg[1].copy()])
    for a, b in zip(singles, pairs):
        assert _bits_equal(a, b)


def test_mtp_stream_equals_greedy_tiny(tiny):
    prompt = list(range(3, 35))
    ids0, st0 = tiny.generate(prompt, 120, mtp=False)
    ids1, st1 = tiny.generate(prompt, 120, mtp=True)
    assert np.array_equal(ids0, ids1)
    assert st1["mtp_steps"] > 0
    ids2, _ = tiny.generate(prompt, 120, mtp=False)
    assert np.array_equal(ids0, ids2)  # deterministic


def _forced(prompt, ids, pattern, n_vocab):
    """Candidates by position: the greedy token (accepted) or a wrong one (rejected) per `pattern(p)`."""
    seq = list(prompt) + [int(t) for t in ids]
    return [seq[p] if pattern(p) else (seq[p] + 1) % n_vocab for p in range(len(seq))]


@pytest.mark.parametrize("mode", ["graph", "persistent"])
def test_mtp_accept_branch_forced(cuda, mode):
    """The accept branch (src/qwythos.cpp:3211-3222: emit c0 and c1, pos += 2, the no-head draft at pos - 1,
    the next draft from column 1) driven by forced candidates taken from the greedy stream: acceptance
    1.0 and alternating accept / reject both reproduce the greedy stream, with the accepted count equal
    to the forced one; both executors emit the same bits."""
    from rapier_b200.engine import Engine, config_tiny

    eng = Engine(config_tiny(max_ctx=256, seed=7), mode=mode)
    prompt = list(range(40, 52))
    n = 101
    ids0, _ = eng.generate(prompt, n, mtp=False)
    V = eng.cfg.n_vocab
    # every candidate right: each round verifies one candidate and emits two tokens
    eng.force_candidates(_forced(prompt, ids0, lambda p: True, V))
    ids1, st1 = eng.generate(prompt, n, mtp=True)
    assert np.array_equal(ids0, ids1)
    assert st1["mtp_steps"] > 0 and st1["mtp_accepted"] == st1["mtp_steps"], st1
    assert st1["mtp_steps"] == (n - 1) // 2
    # candidates right at even positions only: rounds alternate with the position parity
    eng.force_candidates(_forced(prompt, ids0, lambda p: p % 2 == 0, V))
    ids2, st2 = eng.generate(prompt, n, mtp=True)
    assert np.array_equal(ids0, ids2)
    assert 0 < st2["mtp_accepted"] < st2["mtp_steps"], st2
    # the count the forcing implies: walk the rounds as the protocol does
    pos, emitted, steps, acc = len(prompt), 1, 0, 0  # after the seed pass: one token emitted, cur at pos
    while emitted < n:
        if emitted >= n - 1:
            emitted += 1
            continue
        steps += 1
        if (pos + 1) % 2 == 0:  # the candidate for pos + 1 was right
            acc += 1
            emitted += 2
            pos += 2
        else:
            emitted += 1
            pos += 1
    assert (st2["mtp_steps"], st2["mtp_accepted"]) == (steps, acc)
    eng.force_candidates(None)
    ids3, st3 = eng.generate(prompt, n, mtp=True)
    assert np.array_equal(ids0, ids3)
    eng.close()


def test_mtp_accept_with_eos_second_token(tiny):
    """An accepted round whose column-1 token is the end-of-sequence id: the run stops after emitting it,
    the MTP stream equals the greedy stream cut at the same token, and the next run continues exactly as
    the greedy session does."""
    prompt = list(range(60, 70))
    V = tiny.cfg.n_vocab
    tiny.session_reset()
    ref, _, _ = tiny.session_run(prompt, 40, mtp=False)
    # with every candidate right, rounds emit (c0, c1) pairs after the first token: index 2 is a c1
    eos = int(ref[2])
    if eos in [int(t) for t in ref[:2]]:
        pytest.skip("the chosen end-of-sequence token also appears earlier in the stream")
    tiny.session_reset()
    g1, _, _ = tiny.session_run(prompt, 40, mtp=False, eos=eos)
    p1 = tiny.session_pos
    g2, _, _ = tiny.session_run([5, 6], 20, mtp=False)  # the end-of-sequence id is not in the context
    tiny.force_candidates(_forced(prompt, ref, lambda p: True, V))
    tiny.session_reset()
    m1, st, _ = tiny.session_run(prompt, 40, mtp=True, eos=eos)
    assert list(m1) == list(g1) and int(m1[-1]) == eos and len(m1) == 3
    assert st["mtp_accepted"] == st["mtp_steps"] == 1
    assert tiny.session_pos == p1 == len(prompt) + 2
    tiny.force_candidates(None)
    m2, _, _ = tiny.session_run([5, 6], 20, mtp=True)
    assert list(m2) == list(g2)
    tiny.session_reset()


def test_generate_matches_teacher_forcing(tiny):
    prompt = [11, 22, 33, 44]
    ids, _ = tiny.generate(prompt, 8, mtp=False)
    tiny.reset()
    seq = list(prompt)
    for pos in range(len(prompt) + 7):
        _, am = tiny.step([seq[pos]], pos, want_logits=False)
        if pos >= len(prompt) - 1:
            assert am[0] == ids[pos - len(prompt) + 1]
            seq.append(am[0])


@pytest.fixture(scope="module")
def nine_b_4layer(cuda):
    """The 9B geometry cut to 4 layers (GDN layers 0-2, attention layer 3) with the full 248320-row
    lm_head and the MTP block, on the engine and in the oracle."""
    from oracle.model import Model
    from rapier_b200.engine import Engine, config_9b

    cfg = config_9b(max_ctx=65600, seed=1)
    cfg.n_layer = 4
    eng = Engine(cfg)
    m = Model(cfg)
    yield eng, m
    eng.close()


@pytest.mark.slow
def test_9b_shape_logits_bitwise_oracle(nine_b_4layer):
    eng, m = nine_b_4layer
    eng.reset()
    m.reset()
    toks = [7, 248319, 123456, 42]
    for pos, t in enumerate(toks):
        logits, am = eng.step([t], pos)
        want = m.forward(t, pos)
        _assert_bits(logits[0], want, f"9B shape, position {pos}")
        assert am[0] == int(np.argmax(want))
    lg, am = eng.draft_step(toks[-1], len(toks))
    _assert_bits(lg, m.draft(toks[-1], len(toks)), "9B draft")


@pytest.mark.slow
def test_9b_shape_after_65536_token_context(nine_b_4layer):
    """A step at position 65536 after the synthetic 65536-token context (rk_engine_session_fill: seeded
    fp16 K/V in the attention layer, seeded GDN states), bit-identical to the oracle given the same fill:
    the attention layer streams 65537 positions in 256-token chunks."""
    eng, m = nine_b_4layer
    n = 65536
    eng.session_fill(n, seed=5)
    m.fill(n, seed=5)
    for i, t in enumerate([99, 1000]):
        logits, am = eng.step([t], n + i)
        want = m.forward(t, n + i)
        _assert_bits(logits[0], want, f"after the {n}-token context, position {n + i}")
        assert am[0] == int(np.argmax(want))


@pytest.mark.slow
def test_mtp_stream_equals_greedy_9b(cuda):
    """The exactness invariant on the 9B-shaped model (exact MTP, ctx 512): 400 tokens, MTP == greedy, with
    the draft's own candidates and with every candidate forced right."""
    from rapier_b200.engine import Engine, config_9b

    eng = Engine(config_9b(max_ctx=512, seed=1))
    prompt = list(np.random.default_rng(1).integers(0, 248320, 32))
    ids0, st0 = eng.generate(prompt, 400, mtp=False)
    ids1, st1 = eng.generate(prompt, 400, mtp=True)
    assert np.array_equal(ids0, ids1)
    eng.force_candidates(_forced(prompt, ids0, lambda p: True, 248320))
    ids2, st2 = eng.generate(prompt, 400, mtp=True)
    eng.close()
    assert np.array_equal(ids0, ids2)
    assert st2["mtp_accepted"] == st2["mtp_steps"] > 0
    print("9b mtp steps", st1["mtp_steps"], "accepted", st1["mtp_accepted"], "gen ms", st0["gen_ms"], st1["gen_ms"],
          "forced: steps", st2["mtp_steps"], "gen ms", st2["gen_ms"])
