"""GPU parity of the quantized GEMVs against the CPU oracle, through the C-ABI (rapier_b200.ops).

Bit-exact: Q8_1 bytes of the quantizer, the packed layout, the integer sub-block sums, and the packed
GEMV's fp32 outputs against the oracle's restatement of the packed kernel's summation order
(oracle.mmvq_packed). fp32 outputs are also within RTOL = 1e-3 (tests/_util.py) of the oracle's
restatement of the reference's lane order. Columns of a multi-column call: bitwise equal to single-column
calls (the reference's invariant, src/native_mmvq.cu:902-920).
"""
import numpy as np
import pytest
import torch

from tests._util import assert_bits, assert_close, empty_dev, to_dev, to_np

pytestmark = pytest.mark.gpu

Q6, Q8 = 14, 8


def _weights(oracle, t, n_in, n_out, seed, random_bytes=False):
    if random_bytes:  # the reference harness's style (src/test_res.cpp:24-31) with finite fp16 scales
        rng = np.random.default_rng(seed)
        raw = rng.integers(0, 256, size=oracle.weight_bytes(t, n_in, n_out), dtype=np.uint8)
        if t == Q6:
            blk = raw.reshape(-1, 210)
            blk[:, 208:210] = (rng.standard_normal(blk.shape[0]) * 0.01).astype(np.float16).view(np.uint8).reshape(-1, 2)
        else:
            blk = raw.reshape(-1, 34)
            blk[:, 0:2] = (rng.standard_normal(blk.shape[0]) * 0.01).astype(np.float16).view(np.uint8).reshape(-1, 2)
        return raw
    w = oracle.synth_normal(seed, n_in * n_out, std=0.02)
    return oracle.quantize_weights(t, w, n_in, n_out)


def _act(oracle, n_in, ncols, seed):
    x = oracle.synth_normal(seed, n_in * ncols, std=1.0)
    return x, oracle.quantize_q8_1(x, n_in, ncols)


@pytest.mark.parametrize("n_in,ncols", [(4096, 1), (12288, 2), (256, 3), (8192, 16)])
def test_quantize_q8_1_bit_exact(cuda, oracle, n_in, ncols):
    from rapier_b200 import ops

    x, want = _act(oracle, n_in, ncols, 11 + ncols)
    x[5] = 0.0
    if n_in >= 64:
        x[32:64] = 0.0  # an all-zero block
    want = oracle.quantize_q8_1(x, n_in, ncols)
    dx = to_dev(x)
    dq = empty_dev(ops.native_q8_1_bytes(n_in, ncols), torch.uint8)
    ops.native_quantize_q8_1(dx, dq, n_in, ncols)
    assert np.array_equal(to_np(dq), want)


@pytest.mark.parametrize("t", [Q6, Q8])
def test_pack_matches_oracle_and_roundtrips(cuda, oracle, t):
    from rapier_b200 import ops

    n_in, n_out = 4096, 64
    raw = _weights(oracle, t, n_in, n_out, 3, random_bytes=True)
    draw = to_dev(raw)
    dp = empty_dev(ops.packed_bytes(t, n_in, n_out), torch.uint8)
    ops.pack_weights(t, draw, dp, n_in, n_out)
    assert np.array_equal(to_np(dp), oracle.pack_weights(t, raw, n_in, n_out))
    du = empty_dev(raw.size, torch.uint8)
    ops.unpack_weights(t, dp, du, n_in, n_out)
    assert np.array_equal(to_np(du), raw)


@pytest.mark.parametrize("t", [Q6, Q8])
@pytest.mark.parametrize("ncols", [1, 2])
def test_integer_sums_bit_exact(cuda, oracle, t, ncols):
    from rapier_b200 import ops

    n_in, n_out = 4096, 32
    raw = _weights(oracle, t, n_in, n_out, 5 + ncols, random_bytes=True)
    _, xq = _act(oracle, n_in, ncols, 21)
    packed = oracle.pack_weights(t, raw, n_in, n_out)
    nsub = n_in // 16 if t == Q6 else n_in // 32
    out = empty_dev(ncols * n_out * nsub, torch.int32)
    ops.mmvq_isums(t, to_dev(packed), to_dev(xq), out, n_in, n_out, ncols)
    assert np.array_equal(to_np(out), oracle.mmvq_isums(t, raw, xq, n_in, n_out, ncols))


@pytest.mark.parametrize("t", [Q6, Q8])
@pytest.mark.parametrize("shape", [(4096, 12288), (4096, 64), (12288, 4096), (8192, 4096), (1024, 4)])
def test_packed_gemv_vs_oracle(cuda, oracle, t, shape):
    from rapier_b200 import ops

    n_in, n_out = shape
    raw = _weights(oracle, t, n_in, n_out, n_in + n_out)
    _, xq = _act(oracle, n_in, 2, 7)
    want = oracle.mmvq(t, raw, xq, n_in, n_out, 2)
    dp = to_dev(oracle.pack_weights(t, raw, n_in, n_out))
    dx = to_dev(xq)
    y2 = empty_dev(2 * n_out, torch.float32)
    ops.mmvq_packed(t, dp, dx, y2, n_in, n_out, 2)
    assert_close(to_np(y2), want, what=f"packed gemv {t} {shape}")
    assert_bits(to_np(y2), oracle.mmvq_packed(t, raw, xq, n_in, n_out, 2), what=f"packed gemv {t} {shape}")
    # each column of the 2-column call is bitwise the single-column call
    y1 = empty_dev(n_out, torch.float32)
    xcol = ops.native_q8_1_bytes(n_in, 1)
    for j in range(2):
        ops.mmvq_packed(t, dp, dx[j * xcol:], y1, n_in, n_out, 1)
        assert np.array_equal(to_np(y1).view(np.uint32), to_np(y2)[j * n_out:(j + 1) * n_out].view(np.uint32))


@pytest.mark.parametrize("ncols", [3, 4, 5, 8, 16])
def test_packed_gemv_many_columns_bitwise(cuda, oracle, ncols):
    from rapier_b200 import ops

    n_in, n_out = 4096, 256
    raw = _weights(oracle, Q6, n_in, n_out, 99)
    _, xq = _act(oracle, n_in, ncols, 8)
    dp, dx = to_dev(oracle.pack_weights(Q6, raw, n_in, n_out)), to_dev(xq)
    yn = empty_dev(ncols * n_out, torch.float32)
    ops.mmvq_packed(Q6, dp, dx, yn, n_in, n_out, ncols)
    got = to_np(yn)
    assert_close(got, oracle.mmvq(Q6, raw, xq, n_in, n_out, ncols), what="many columns")
    assert_bits(got, oracle.mmvq_packed(Q6, raw, xq, n_in, n_out, ncols), what="many columns")
    y1 = empty_dev(n_out, torch.float32)
    xcol = ops.native_q8_1_bytes(n_in, 1)
    for j in range(ncols):
        ops.mmvq_packed(Q6, dp, dx[j * xcol:], y1, n_in, n_out, 1)
        assert np.array_equal(to_np(y1).view(np.uint32), got[j * n_out:(j + 1) * n_out].view(np.uint32))


@pytest.mark.parametrize("t", [Q6, Q8])
@pytest.mark.parametrize("ncols", [1, 2])
def test_packed_res_epilogue(cuda, oracle, t, ncols):
    """rk_mmvq_packed_res == plain GEMV + residual add (and the 4-row sum-of-squares partials), within
    the reference harness's 1e-3 (src/test_res.cpp:68, :103, :108-112); y == res in place."""
    from rapier_b200 import ops

    n_in, n_out = 12288, 4096
    raw = _weights(oracle, t, n_in, n_out, 77)
    _, xq = _act(oracle, n_in, ncols, 3)
    res = oracle.synth_normal(4, n_out * ncols, std=1.0)
    want_y, want_p = oracle.mmvq_res(t, raw, xq, res, n_in, n_out, ncols)
    dp, dx = to_dev(oracle.pack_weights(t, raw, n_in, n_out)), to_dev(xq)
    dy = to_dev(res.copy())
    part = empty_dev(ncols * n_out // 4, torch.float32)
    ops.mmvq_packed_res(t, dp, dx, dy, dy, part, n_in, n_out, ncols)
    assert_close(to_np(dy), want_y, what="res y")
    assert_close(to_np(part), want_p, what="res partials")
    py, pp = oracle.mmvq_packed(t, raw, xq, n_in, n_out, ncols, res=res)
    assert_bits(to_np(dy), py, what="res y")
    assert_bits(to_np(part), pp, what="res partials")


@pytest.mark.parametrize("t", [Q6, Q8])
@pytest.mark.parametrize("shape,ncols", [((4096, 1000), 1), ((2048, 333), 2), ((4352, 96), 5)])
def test_gguf_layout_gemv(cuda, oracle, t, shape, ncols):
    """The drop-in rk_mmvq on unrepacked GGUF rows (ragged n_out, n_in not a multiple of 1024)."""
    from rapier_b200 import ops

    n_in, n_out = shape
    if t == Q6 and n_in % 256:
        pytest.skip("Q6_K needs n_in % 256 == 0")
    raw = _weights(oracle, t, n_in, n_out, 5)
    _, xq = _act(oracle, n_in, ncols, 6)
    y = empty_dev(ncols * n_out, torch.float32)
    ops.native_mmvq(t, to_dev(raw), to_dev(xq), y, n_in, n_out, ncols)
    assert_close(to_np(y), oracle.mmvq(t, raw, xq, n_in, n_out, ncols), what="gguf layout")


@pytest.mark.parametrize("t", [Q6, Q8])
def test_gguf_layout_res(cuda, oracle, t):
    from rapier_b200 import ops

    n_in, n_out = 4096, 4095  # ragged last partial slot
    raw = _weights(oracle, t, n_in, n_out, 15)
    _, xq = _act(oracle, n_in, 1, 16)
    res = oracle.synth_normal(17, n_out, std=1.0)
    want_y, want_p = oracle.mmvq_res(t, raw, xq, res, n_in, n_out, 1)
    dy = to_dev(res.copy())
    part = empty_dev((n_out + 3) // 4, torch.float32)
    ops.native_q6_k_mmvq_res(to_dev(raw), to_dev(xq), dy, dy, part, n_in, n_out) if t == Q6 else \
        ops.native_q8_0_mmvq_res(to_dev(raw), to_dev(xq), dy, dy, part, n_in, n_out)
    assert_close(to_np(dy), want_y, what="gguf res y")
    assert_close(to_np(part), want_p, what="gguf res partials")


def test_config1_full_shape(cuda, oracle):
    """The single-GEMV workload: W 12288x4096 ~ N(0, 0.02) -> Q6_K, x ~ N(0, 1) -> Q8_1, ncols 1 and 2."""
    from rapier_b200 import ops

    n_in, n_out = 4096, 12288
    raw = _weights(oracle, Q6, n_in, n_out, 1)
    x, xq = _act(oracle, n_in, 2, 2)
    dx = to_dev(x)
    dq = empty_dev(ops.native_q8_1_bytes(n_in, 2), torch.uint8)
    ops.native_quantize_q8_1(dx, dq, n_in, 2)
    assert np.array_equal(to_np(dq), xq)
    dp = empty_dev(ops.packed_bytes(Q6, n_in, n_out), torch.uint8)
    ops.pack_weights(Q6, to_dev(raw), dp, n_in, n_out)
    y = empty_dev(2 * n_out, torch.float32)
    ops.mmvq_packed(Q6, dp, dq, y, n_in, n_out, 2)
    want = oracle.mmvq(Q6, raw, xq, n_in, n_out, 2)
    assert_close(to_np(y), want, what="config 1")
    assert_bits(to_np(y), oracle.mmvq_packed(Q6, raw, xq, n_in, n_out, 2), what="config 1")
    # against the float64 product of the dequantized operands (scale of the quantization error)
    wd = oracle.dequantize_weights(Q6, raw, n_in, n_out).reshape(n_out, n_in).astype(np.float64)
    xd = oracle.dequantize_q8_1(xq, 2 * n_in).reshape(2, n_in).astype(np.float64)
    y64 = (wd @ xd.T).T.ravel()
    assert np.max(np.abs(to_np(y) - y64)) <= 1e-4 * np.max(np.abs(y64))
    assert ops.device_status() == 0
