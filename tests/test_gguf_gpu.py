"""The GGUF loader end to end on the GPU: a synthetic engine's model written as a qwen35 GGUF file
(rapier_b200.gguf_export, gguf-py) and loaded back with rk_engine_create_gguf gives the same logits bit for
bit and the same greedy / MTP token streams; a matrix of a type the engine has no GEMV for is refused."""
import numpy as np
import pytest

gguf = pytest.importorskip("gguf")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def pair(tmp_path_factory):
    from rapier_b200.engine import Engine, config_tiny
    from rapier_b200.gguf_export import export_gguf

    path = tmp_path_factory.mktemp("gguf") / "tiny.gguf"
    syn = Engine(config_tiny(max_ctx=256))
    export_gguf(syn, str(path))
    fil = Engine.from_gguf(str(path), max_ctx=256)
    yield syn, fil, path
    fil.close()
    syn.close()


def test_config_round_trip(pair):
    syn, fil, _ = pair
    for f in ("n_layer", "n_embd", "n_ff", "n_vocab", "ssm_h_k", "ssm_h_v", "n_head", "n_head_kv", "n_rot",
              "attn_interval", "has_mtp", "max_ctx"):
        assert getattr(fil.cfg, f) == getattr(syn.cfg, f), f
    assert np.float32(fil.cfg.eps) == np.float32(syn.cfg.eps) and fil.cfg.rope_base == syn.cfg.rope_base


def test_tensors_and_logits_bitwise(pair):
    from rapier_b200 import engine as E

    syn, fil, _ = pair
    for tid in (E.T_TOK_EMBD, E.T_OUTPUT, E.T_EH_PROJ, E.layer_tid(0, E.L_GDN_QKV), E.layer_tid(3, E.L_ATT_Q)):
        assert np.array_equal(syn.read_tensor(tid), fil.read_tensor(tid)), tid
    syn.reset()
    fil.reset()
    for pos, tok in enumerate([5, 900, 17, 4000, 3]):
        (la, ta), (lb, tb) = syn.step([tok], pos), fil.step([tok], pos)
        assert np.array_equal(la, lb) and ta == tb, pos


@pytest.mark.parametrize("mtp", [False, True])
def test_generation_equal(pair, mtp):
    syn, fil, _ = pair
    prompt = list(range(40, 72))
    a, _ = syn.generate(prompt, 48, mtp=mtp)
    b, _ = fil.generate(prompt, 48, mtp=mtp)
    assert list(a) == list(b)


def test_other_matrix_type_refused(pair, tmp_path):
    from rapier_b200 import _lib
    from rapier_b200.engine import Engine

    _, _, path = pair
    r = gguf.GGUFReader(str(path))
    w = gguf.GGUFWriter(str(tmp_path / "f32.gguf"), "qwen35")
    for f in r.fields.values():
        if f.name.startswith("qwen35."):
            v = f.parts[f.data[0]]
            (w.add_uint32 if v.dtype == np.uint32 else w.add_float64 if v.dtype == np.float64 else w.add_float32)(
                f.name, v[0].item())
    for t in r.tensors:
        if t.name == "blk.0.ffn_up.weight":  # the one matrix stored as F32: no GEMV for it
            w.add_tensor(t.name, np.zeros((int(t.shape[1]), int(t.shape[0])), np.float32))
        elif t.tensor_type == gguf.GGMLQuantizationType.Q6_K:
            w.add_tensor(t.name, np.array(t.data), raw_dtype=t.tensor_type)
        else:
            w.add_tensor(t.name, np.array(t.data).reshape([int(d) for d in reversed(t.shape)]))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with pytest.raises(_lib.RkError) as ei:
        Engine.from_gguf(str(tmp_path / "f32.gguf"), max_ctx=256)
    assert ei.value.code == _lib.RK_EUNSUPPORTED
