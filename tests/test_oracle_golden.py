"""Pins the CPU oracle against the golden vectors made from gguf-py 0.19.0 (tests/golden/make_golden.py)
and against numpy, before it is trusted as the checker of the CUDA kernels. CPU only."""
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(__file__), "golden", "ggml_formats.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def test_f16_conversion_matches_numpy(oracle):
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(200000) * np.float32(10.0) ** rng.integers(-9, 6, 200000)).astype(np.float32)
    edge = np.array([0.0, -0.0, 65504, 65519.99, 65520, 1e-8, 2 ** -24, 2 ** -25, 2 ** -25 * 1.0001, 2 ** -14,
                     np.inf, -np.inf, 6.1e-5, 5.96e-8], np.float32)
    x = np.concatenate([x, edge])
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(oracle.f32_to_f16(x), want)
    allh = np.arange(65536, dtype=np.uint16)
    got = oracle.f16_to_f32(allh)
    ref = allh.view(np.float16).astype(np.float32)
    same = (got.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(got) & np.isnan(ref))
    assert same.all()


def test_q6k_dequant_matches_gguf(oracle, gold):
    n_in, n_out = int(gold["n_in"]), int(gold["n_out"])
    got = oracle.dequantize_weights(oracle.TYPE_Q6_K, gold["q6k_raw"], n_in, n_out)
    assert np.array_equal(got.view(np.uint32), gold["q6k_deq"].view(np.uint32))


def test_q80_encode_matches_gguf(oracle, gold):
    n_in, n_out = int(gold["n_in"]), int(gold["n_out"])
    got = oracle.quantize_weights(oracle.TYPE_Q8_0, gold["q80_src"], n_in, n_out)
    assert np.array_equal(got, gold["q80_raw"])


@pytest.mark.parametrize("kind", ["q6k", "q80"])
def test_integer_subblock_sums_match_gguf_codes(oracle, gold, kind):
    """The restated dp4a dot (q6_q8_dot_impl / small_q8_dot) gives exactly the integer sums computed from
    gguf-decoded codes."""
    n_in, n_out, nc = int(gold["n_in"]), int(gold["n_out"]), int(gold["ncols"])
    t = oracle.TYPE_Q6_K if kind == "q6k" else oracle.TYPE_Q8_0
    w = gold["q6k_raw"] if kind == "q6k" else gold["q80_raw"]
    got = oracle.mmvq_isums(t, w, gold["xq"], n_in, n_out, nc)
    assert np.array_equal(got, gold[f"{kind}_isums"])


def test_gemv_equals_integer_sums_times_scales(oracle, gold):
    """The fp32 GEMV is the scaled sum of the pinned integer sums (float64 reconstruction)."""
    n_in, n_out, nc = int(gold["n_in"]), int(gold["n_out"]), int(gold["ncols"])
    y = oracle.mmvq(oracle.TYPE_Q6_K, gold["q6k_raw"], gold["xq"], n_in, n_out, nc).reshape(nc, n_out)
    isums = gold["q6k_isums"].reshape(nc, n_out, n_in // 16).astype(np.float64)
    raw = gold["q6k_raw"].reshape(n_out, n_in // 256, 210)
    d = raw[:, :, 208:210].copy().view(np.float16).astype(np.float64).reshape(n_out, n_in // 256)
    d_sub = np.repeat(d, 16, axis=1)
    xd = gold["xq_d"].view(np.float16).astype(np.float64).reshape(nc, n_in // 32)
    xd_sub = np.repeat(xd, 2, axis=1)
    want = (isums * d_sub[None] * xd_sub[:, None, :]).sum(axis=-1)
    assert np.max(np.abs(y - want)) <= 1e-4 * np.max(np.abs(want))


def test_q6k_encoder_roundtrip_and_gguf_decode(oracle):
    import gguf
    from gguf import GGMLQuantizationType as T

    n_in, n_out = 1024, 16
    w = oracle.synth_normal(5, n_in * n_out, std=0.02)
    q = oracle.quantize_weights(oracle.TYPE_Q6_K, w, n_in, n_out)
    deq = oracle.dequantize_weights(oracle.TYPE_Q6_K, q, n_in, n_out)
    assert np.array_equal(deq, gguf.quants.dequantize(q.reshape(n_out, -1), T.Q6_K).ravel())
    rel = np.sqrt(np.mean((deq - w) ** 2)) / np.sqrt(np.mean(w ** 2))
    assert rel < 0.03


@pytest.mark.parametrize("t", [14, 8])
def test_pack_unpack_roundtrip(oracle, t):
    rng = np.random.default_rng(t)
    n_in, n_out = 3072, 12
    raw = rng.integers(0, 256, size=oracle.weight_bytes(t, n_in, n_out), dtype=np.uint8)
    p = oracle.pack_weights(t, raw, n_in, n_out)
    assert p.size == raw.size
    assert np.array_equal(oracle.unpack_weights(t, p, n_in, n_out), raw)


def test_pack_rejects_unaligned_shapes(oracle):
    raw = np.zeros(oracle.weight_bytes(14, 768, 4), np.uint8)
    with pytest.raises(ValueError):
        oracle.pack_weights(14, raw, 768, 4)


def test_synth_generator_matches_numpy_restatement(oracle):
    seed, n = 1234, 4096
    M = (1 << 64) - 1
    idx = np.arange(n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed) * np.uint64(0x9E3779B97F4A7C15) + idx + np.uint64(0x632BE59BD9B4E019)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    s = sum(((z >> np.uint64(16 * k)) & np.uint64(0xFFFF)).astype(np.int64) for k in range(4)) - 131070
    scale = np.float32(oracle.synth_scale(0.5))
    want = (s.astype(np.float32) * scale + np.float32(0.25)).astype(np.float32)
    got = oracle.synth_normal(seed, n, std=0.5, mean=0.25)
    assert np.array_equal(got, want)
    big = oracle.synth_normal(7, 1 << 20, std=0.02)
    assert abs(big.std() - 0.02) < 2e-4 and abs(big.mean()) < 2e-4
    del M


def test_q8_1_rules(oracle):
    x = np.zeros(96, np.float32)
    x[32:64] = np.linspace(-3, 3, 32, dtype=np.float32)
    x[64] = np.inf
    q = oracle.quantize_q8_1(x, 96, 1).reshape(3, 36)
    assert np.all(q[0] == 0)  # all-zero block: d = 0, codes 0
    d = q[1, 0:2].copy().view(np.float16)[0]
    assert np.isclose(float(d), 3 / 127, rtol=1e-3)
    codes = q[1, 4:].view(np.int8)
    assert codes.min() == -127 and codes.max() == 127
    d2 = q[2, 0:2].copy().view(np.float16)[0]
    assert float(d2) == 65504.0  # non-finite d clamped to the fp16 maximum


def test_gdn_oracle_matches_unfused_restatement(oracle):
    """The fused GDN step restated from src/fused_gdn.cu:39-111 agrees with a float64 restatement of the
    unfused chain of src/gdn.cu:46-170 (decay, update, read-out, q-scale, gated RMSNorm)."""
    rng = np.random.default_rng(3)
    h_k, h_v, S = 4, 8, 128
    state = (rng.standard_normal((S, h_v, S)) * 0.01).astype(np.float32)
    q = rng.standard_normal(h_k * S).astype(np.float32)
    k = rng.standard_normal(h_k * S).astype(np.float32)
    q /= np.linalg.norm(q.reshape(h_k, S), axis=1).repeat(S)
    k /= np.linalg.norm(k.reshape(h_k, S), axis=1).repeat(S)
    v = rng.standard_normal(h_v * S).astype(np.float32)
    gate = -np.abs(rng.standard_normal(h_v)).astype(np.float32)
    beta = (1 / (1 + np.exp(-rng.standard_normal(h_v)))).astype(np.float32)
    z = rng.standard_normal(h_v * S).astype(np.float32)
    gamma = (1 + 0.1 * rng.standard_normal(S)).astype(np.float32)
    eps = 1e-6
    st2, y, q8 = oracle.gdn_step_norm_silu_q8(state, q, k, v, gate, beta, z, gamma, eps, h_k, h_v)
    s64 = state.astype(np.float64).copy()
    y64 = np.zeros(h_v * S)
    for h in range(h_v):
        kk = k[(h % h_k) * S:(h % h_k + 1) * S].astype(np.float64)
        qq = q[(h % h_k) * S:(h % h_k + 1) * S].astype(np.float64)
        dec = np.exp(gate[h])
        Sh = s64[:, h, :] * dec
        delta = (v[h * S:(h + 1) * S] - kk @ Sh) * beta[h]
        Sh = Sh + np.outer(kk, delta)
        s64[:, h, :] = Sh
        o = (qq @ Sh) / np.sqrt(S)
        inv = 1 / np.sqrt(np.mean(o * o) + eps)
        zz = z[h * S:(h + 1) * S]
        y64[h * S:(h + 1) * S] = o * inv * gamma * zz / (1 + np.exp(-zz))
    assert np.max(np.abs(st2 - s64)) < 1e-5
    assert np.max(np.abs(y - y64)) < 1e-4 * np.max(np.abs(y64))


@pytest.mark.parametrize("ncols", [1, 2])
def test_flash_order_attention_matches_reference_form(oracle, ncols):
    """The attention restated in the decode engine's flash-decode order (chunks, per-chunk softmax, combine)
    agrees with the reference-form restatement (one softmax over all tokens, float64 sums) within fp32
    rounding, at chunk boundaries and over several chunks; column c attends 0..pos+c."""
    nh, nkv, HD, n_rot, eps = 16, 4, 256, 64, 1e-6
    max_ctx = 300
    rope = oracle.rope_table(max_ctx, n_rot, 1e7)
    qn = oracle.synth_normal(11, HD, std=0.02, mean=1.0)
    kn = oracle.synth_normal(12, HD, std=0.02, mean=1.0)
    kc = np.zeros((max_ctx, nkv, HD), np.uint16)
    vc = np.zeros_like(kc)
    stride = nh * 2 * HD + 2 * nkv * HD
    for pos in range(0, 260, ncols):
        proj = oracle.synth_normal(100 + pos, ncols * stride)
        o, q8 = oracle.attn_flash_f16(proj, ncols, stride, qn, kn, rope, n_rot, nh, nkv, kc, vc, pos, 32, eps)
        if pos % 31 and pos not in (32, 64, 256):
            continue
        for c in range(ncols):
            col = proj[c * stride:(c + 1) * stride]
            q, g = oracle.split_qg(col[:nh * 2 * HD], nh, HD)
            q = oracle.rope_apply(oracle.rms_norm_rows(q, qn, nh, HD, eps), nh, HD, n_rot, rope, pos + c)
            want = oracle.gqa_decode_f16(q, kc.ravel(), vc.ravel(), nh, nkv, HD, pos + c + 1, 0.0625)
            got = o[c * nh * HD:(c + 1) * nh * HD]
            assert np.max(np.abs(got - want)) <= 2e-6 * np.max(np.abs(want)), (pos, c)
            assert np.array_equal(q8[c * nh * 8 * 36:(c + 1) * nh * 8 * 36],
                                  oracle.sigmul_q8_1(got, g))


@pytest.mark.parametrize("t", [14, 8])
def test_packed_order_gemv_matches_reference_order(oracle, t):
    """The GEMV in the packed kernel's summation order uses the same integer sums as the reference's lane
    order; the fp32 results differ only by rounding (a few ulp of the row's scale)."""
    n_in, n_out = 8192, 96
    raw = oracle.quantize_weights(t, oracle.synth_normal(31, n_in * n_out, std=0.02), n_in, n_out)
    xq = oracle.quantize_q8_1(oracle.synth_normal(32, n_in * 2), n_in, 2)
    a = oracle.mmvq(t, raw, xq, n_in, n_out, 2)
    b = oracle.mmvq_packed(t, raw, xq, n_in, n_out, 2)
    assert np.max(np.abs(a - b)) <= 1e-6 * np.max(np.abs(a))
    res = oracle.synth_normal(33, 2 * n_out)
    y, p = oracle.mmvq_packed(t, raw, xq, n_in, n_out, 2, res=res)
    assert np.array_equal(y, b + res)
    assert np.array_equal(p, np.concatenate([oracle.row_sumsq_partials(y[:n_out]), oracle.row_sumsq_partials(y[n_out:])]))
