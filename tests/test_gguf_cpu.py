"""The GGUF side of the model loader, on the CPU: rk_gguf_model_config on qwen35 files written here with
gguf-py (the geometry from the tensor shapes and metadata, as the reference's load_model reads them,
src/qwythos.cpp:1978-2016), refusals (another architecture, a truncated file, a bad magic), and the RoPE
table the engine builds: plain NEOX equals the oracle's table, YaRN equals a float64 restatement of the
published formula with the reference's parameters (ext 1, attn 1, beta_fast 32, beta_slow 1)."""
import ctypes as C
import math

import numpy as np
import pytest

gguf = pytest.importorskip("gguf")


def _tiny_gguf(path, arch="qwen35", yarn=None):
    """A 2-layer qwen35 file (1 GDN + 1 attention layer, an MTP block) of random Q6_K bytes."""
    H, FF, V, S, hk, hv, nh, nkv = 1024, 2048, 512, 128, 4, 8, 4, 1
    rng = np.random.default_rng(0)
    w = gguf.GGUFWriter(str(path), arch)
    w.add_uint32(f"{arch}.block_count", 3)
    w.add_uint32(f"{arch}.nextn_predict_layers", 1)
    w.add_uint32(f"{arch}.rope.dimension_count", 64)
    w.add_float64(f"{arch}.rope.freq_base", 1e7)
    w.add_float32(f"{arch}.attention.layer_norm_rms_epsilon", 1e-6)
    if yarn:
        w.add_float32(f"{arch}.rope.scaling.factor", yarn[0])
        w.add_uint32(f"{arch}.rope.scaling.original_context_length", yarn[1])

    def q6(name, n_out, n_in):
        raw = rng.integers(0, 256, size=(n_out, n_in // 256 * 210), dtype=np.uint8)
        w.add_tensor(name, raw, raw_dtype=gguf.GGMLQuantizationType.Q6_K)

    def f32(name, *shape):
        w.add_tensor(name, np.ones(shape, np.float32))

    q6("token_embd.weight", V, H)
    q6("output.weight", V, H)
    f32("output_norm.weight", H)
    for il, kind in enumerate(["gdn", "att", "att"]):
        b = f"blk.{il}."
        f32(b + "attn_norm.weight", H)
        f32(b + "post_attention_norm.weight", H)
        q6(b + "ffn_up.weight", FF, H)
        q6(b + "ffn_gate.weight", FF, H)
        q6(b + "ffn_down.weight", H, FF)
        if kind == "gdn":
            q6(b + "attn_qkv.weight", 2 * hk * S + hv * S, H)
            q6(b + "attn_gate.weight", hv * S, H)
            q6(b + "ssm_beta.weight", hv, H)
            q6(b + "ssm_alpha.weight", hv, H)
            q6(b + "ssm_out.weight", H, hv * S)
            f32(b + "ssm_conv1d.weight", 2 * hk * S + hv * S, 4)
            f32(b + "ssm_a", hv)
            f32(b + "ssm_dt.bias", hv)
            f32(b + "ssm_norm.weight", S)
        else:
            q6(b + "attn_q.weight", 2 * nh * 256, H)
            q6(b + "attn_k.weight", nkv * 256, H)
            q6(b + "attn_v.weight", nkv * 256, H)
            q6(b + "attn_output.weight", H, nh * 256)
            f32(b + "attn_q_norm.weight", 256)
            f32(b + "attn_k_norm.weight", 256)
    q6("blk.2.nextn.eh_proj.weight", H, 2 * H)
    for n in ("enorm", "hnorm", "shared_head_norm"):
        f32(f"blk.2.nextn.{n}.weight", H)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def _config(path, max_ctx=256):
    from rapier_b200 import _lib

    c = _lib.ModelConfig()
    rc = _lib.lib().rk_gguf_model_config(str(path).encode(), max_ctx, C.byref(c))
    return rc, c


def test_model_config_from_tensor_shapes(tmp_path):
    p = tmp_path / "m.gguf"
    _tiny_gguf(p)
    rc, c = _config(p)
    assert rc == 0
    got = (c.n_layer, c.n_embd, c.n_ff, c.n_vocab, c.ssm_h_k, c.ssm_h_v, c.n_head, c.n_head_kv, c.n_rot,
           c.attn_interval, c.has_mtp, c.max_ctx)
    assert got == (2, 1024, 2048, 512, 4, 8, 4, 1, 64, 2, 1, 256)
    assert c.eps == np.float32(1e-6) and c.rope_base == 1e7 and c.rope_yarn_factor == 1.0


def test_model_config_reads_yarn(tmp_path):
    p = tmp_path / "y.gguf"
    _tiny_gguf(p, yarn=(4.0, 65536))
    rc, c = _config(p)
    assert rc == 0 and c.rope_yarn_factor == 4.0 and c.rope_orig_ctx == 65536


def test_refusals(tmp_path):
    from rapier_b200 import _lib

    p = tmp_path / "other.gguf"
    _tiny_gguf(p, arch="llama")
    assert _config(p)[0] == _lib.RK_EUNSUPPORTED
    good = tmp_path / "m.gguf"
    _tiny_gguf(good)
    data = good.read_bytes()
    (tmp_path / "cut.gguf").write_bytes(data[: len(data) // 2])
    assert _config(tmp_path / "cut.gguf")[0] == _lib.RK_EINVAL
    (tmp_path / "magic.gguf").write_bytes(b"GGML" + data[4:])
    assert _config(tmp_path / "magic.gguf")[0] == _lib.RK_EINVAL
    assert _config(tmp_path / "missing.gguf")[0] == _lib.RK_EINVAL


@pytest.mark.parametrize("ne1", [0, 2**63 + 5, 2**41])
def test_refuses_bad_tensor_dims(tmp_path, ne1):
    """A tensor directory entry with a zero, negative-as-int64 or absurd dimension is refused (the byte
    count is computed in exact integer arithmetic, so no overflow lets a tensor pass the end-of-file check)."""
    from rapier_b200 import _lib

    good = tmp_path / "m.gguf"
    _tiny_gguf(good)
    data = bytearray(good.read_bytes())
    name = b"token_embd.weight"
    at = data.index(name) + len(name)  # the directory entry: n_dims u32, ne[0] u64, ne[1] u64, ...
    assert int.from_bytes(data[at:at + 4], "little") == 2
    data[at + 12:at + 20] = int(ne1).to_bytes(8, "little")
    bad = tmp_path / "dims.gguf"
    bad.write_bytes(bytes(data))
    assert _config(bad)[0] == _lib.RK_EINVAL


def _table(n_rot, base, factor, orig, n_pos):
    from rapier_b200 import _lib

    out = np.empty(n_pos * n_rot, np.float32)
    assert _lib.lib().rk_rope_table(n_rot, base, factor, orig, n_pos, out.ctypes.data_as(C.c_void_p)) == 0
    return out.reshape(n_pos, n_rot // 2, 2)


def test_rope_table_plain_matches_oracle(oracle):
    got = _table(64, 1e7, 1.0, 262144, 300)
    want = oracle.rope_table(300, 64, 1e7).reshape(300, 32, 2)
    assert np.array_equal(got, want)


def test_rope_table_yarn_restated():
    n_rot, base, factor, orig, n_pos = 64, 1e7, 4.0, 65536, 200
    got = _table(n_rot, base, factor, orig, n_pos).astype(np.float64)

    def corr_dim(beta):
        return n_rot * math.log(orig / (beta * 2 * math.pi)) / (2 * math.log(base))

    lo, hi = max(0.0, math.floor(corr_dim(32.0))), min(n_rot - 1.0, math.ceil(corr_dim(1.0)))
    mscale = 1 + 0.1 * math.log(factor)
    i = np.arange(n_rot // 2)
    ramp = 1 - np.clip((i - lo) / max(0.001, hi - lo), 0, 1)
    ext = np.arange(n_pos)[:, None] * base ** (-2.0 * i / n_rot)[None, :]
    a = ext / factor * (1 - ramp) + ext * ramp
    assert np.allclose(got[..., 0], np.cos(a) * mscale, atol=1e-6)
    assert np.allclose(got[..., 1], np.sin(a) * mscale, atol=1e-6)
    assert not np.allclose(got, _table(n_rot, base, 1.0, orig, n_pos))  # scaling changes the table
