"""Q5_K / Q4_K (the K-quants of the reference's Q5_K_M build) in the CPU oracle, pinned without a GPU: the
oracle's block decode equals gguf-py's dequantizer bit for bit; the oracle's GEMV (the reference's per-thread
vec_dot_q5_K_q8_1 / _q4_K_q8_1 expression and reduction order) matches the dot of the dequantized weights with
the dequantized Q8_1 activations; its integer sums rebuild that dot exactly; the C-ABI's byte counts."""
import numpy as np
import pytest

gguf = pytest.importorskip("gguf")

KQ = {13: "Q5_K", 12: "Q4_K"}


@pytest.mark.parametrize("t", [13, 12])
def test_decode_matches_gguf_py(oracle, t):
    w = oracle.random_kquant_weights(t, 2048, 6, 3)
    mine = oracle.dequant_kq(t, w, 2048 * 6)
    ref = gguf.quants.dequantize(w.reshape(6, -1), getattr(gguf.GGMLQuantizationType, KQ[t])).reshape(-1)
    assert np.array_equal(mine, ref.astype(np.float32))


def _q8_values(oracle, xq, n):
    b = xq.reshape(-1, 36)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float64).reshape(-1, 1)
    return (b[:, 4:].view(np.int8).astype(np.float64) * d).reshape(-1)[:n]


@pytest.mark.parametrize("t", [13, 12])
@pytest.mark.parametrize("n_in,ncols", [(256, 1), (4096, 2), (12288, 1)])
def test_gemv_matches_dequantized_dot(oracle, t, n_in, ncols):
    n_out = 24
    w = oracle.random_kquant_weights(t, n_in, n_out, n_in + t)
    x = oracle.synth_normal(7, n_in * ncols)
    xq = oracle.quantize_q8_1(x, n_in, ncols)
    y = oracle.mmvq(t, w, xq, n_in, n_out, ncols).reshape(ncols, n_out)
    W = oracle.dequant_kq(t, w, n_in * n_out).astype(np.float64).reshape(n_out, n_in)
    for c in range(ncols):
        xv = _q8_values(oracle, xq[c * (n_in // 32) * 36:(c + 1) * (n_in // 32) * 36], n_in)
        want = W @ xv
        np.testing.assert_allclose(y[c], want, rtol=1e-3, atol=1e-3 * np.abs(want).max())


@pytest.mark.parametrize("t", [13, 12])
def test_isums_rebuild_the_dot(oracle, t):
    n_in, n_out = 2048, 8
    w = oracle.random_kquant_weights(t, n_in, n_out, 11)
    xq = oracle.quantize_q8_1(oracle.synth_normal(9, n_in), n_in, 1)
    isums = oracle.mmvq_isums(t, w, xq, n_in, n_out).reshape(n_out, n_in // 32, 2).astype(np.float64)
    bb = 176 if t == 13 else 144
    blk = w.reshape(n_out, n_in // 256, bb)
    d = blk[:, :, 0:2].copy().view(np.float16).astype(np.float64)[..., 0]
    dmin = blk[:, :, 2:4].copy().view(np.float16).astype(np.float64)[..., 0]
    d8 = xq.reshape(-1, 36)[:, 0:2].copy().view(np.float16).astype(np.float64)[:, 0]
    s = isums.reshape(n_out, n_in // 256, 8, 2)
    d8b = d8.reshape(n_in // 256, 8)
    rebuilt = (d * (s[..., 0] * d8b).sum(-1) - dmin * (s[..., 1] * d8b).sum(-1)).sum(-1)
    y = oracle.mmvq(t, w, xq, n_in, n_out)
    np.testing.assert_allclose(y, rebuilt, rtol=1e-4, atol=1e-5 * np.abs(rebuilt).max())


def test_abi_byte_counts():
    from rapier_b200 import _lib

    L = _lib.lib()
    assert L.rk_weight_bytes(13, 4096, 10) == 16 * 176 * 10
    assert L.rk_weight_bytes(12, 4096, 10) == 16 * 144 * 10
    assert L.rk_weight_bytes(13, 4000, 10) == 0  # not a multiple of 256
    assert L.rk_packed_bytes(13, 4096, 12) == 0  # no packed layout for the K-quants
