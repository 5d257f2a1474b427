"""The model oracle stands alone (it imports nothing from the product package): its restated geometry and
synthetic tensor ids equal the engine's, and its pieces run on the CPU (a tiny model's step, draft and
greedy decoding; the engine-order attention at a cache boundary)."""
import numpy as np


def test_oracle_constants_equal_engine():
    from oracle import model as M
    from rapier_b200 import engine as E

    for name in ("T_TOK_EMBD", "T_OUT_NORM", "T_OUTPUT", "T_ENORM", "T_HNORM", "T_EH_PROJ", "T_SHNORM",
                 "L_ATTN_NORM", "L_POST_NORM", "L_FFN_UP", "L_FFN_GATE", "L_FFN_DOWN", "L_GDN_QKV", "L_GDN_Z",
                 "L_GDN_BETA", "L_GDN_ALPHA", "L_GDN_OUT", "L_GDN_CONV", "L_GDN_A", "L_GDN_DT", "L_GDN_NORM",
                 "L_ATT_Q", "L_ATT_K", "L_ATT_V", "L_ATT_O", "L_ATT_QN", "L_ATT_KN"):
        assert getattr(M, name) == getattr(E, name), name
    assert all(M.layer_tid(il, s) == E.layer_tid(il, s) for il in range(40) for s in range(32))
    for mk, ek in ((M.config_9b(512, 3), E.config_9b(512, 3)), (M.config_tiny(64, 5), E.config_tiny(64, 5))):
        for f in ("n_layer", "n_embd", "n_ff", "n_vocab", "ssm_h_k", "ssm_h_v", "n_head", "n_head_kv", "n_rot",
                  "attn_interval", "has_mtp", "max_ctx", "rope_base", "seed"):
            assert getattr(mk, f) == getattr(ek, f), f
        assert np.float32(mk.eps) == np.float32(ek.eps)


def test_oracle_chunk_rule_equals_engine_rule():
    from oracle import oracle as O

    # the rule as the engine states it: the smallest of 32, 64, 128, 256 tokens that splits max_ctx into at
    # most 512 chunks
    for max_ctx, want in ((64, 32), (512, 32), (16384, 32), (16385, 64), (66032, 256), (131072, 256), (200000, 256)):
        assert O.attn_chunk_len(max_ctx) == want, max_ctx


def test_tiny_oracle_runs_and_is_deterministic():
    from oracle.model import Model, config_tiny

    m = Model(config_tiny(max_ctx=64, seed=7))
    a = m.generate([3, 1, 4], 6)
    b = m.generate([3, 1, 4], 6)
    assert a == b and len(a) == 6
    m.reset()
    m.forward(3, 0)
    d = m.draft(1, 1)
    assert d.shape == (m.V,) and np.all(np.isfinite(d))
    assert m.draft(4, 2, with_head=False) is None
