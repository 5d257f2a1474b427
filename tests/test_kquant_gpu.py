"""Q5_K / Q4_K GEMVs on GGUF rows through the C-ABI against the CPU oracle: the integer sub-block sums
(dot1 * scale, dot2 * min of the reference's block threads) bit for bit; y within RTOL = 1e-3 for 1..16
columns; the residual epilogue (y = W x + res and the 4-row sum-of-squares partials); argument checks."""
import numpy as np
import pytest
import torch

from tests._util import assert_close, empty_dev, to_dev, to_np

pytestmark = pytest.mark.gpu


def _case(oracle, t, n_in, n_out, ncols, seed):
    w = oracle.random_kquant_weights(t, n_in, n_out, seed)
    xq = oracle.quantize_q8_1(oracle.synth_normal(seed + 1, n_in * ncols), n_in, ncols)
    return w, xq


@pytest.mark.parametrize("t", [13, 12])
@pytest.mark.parametrize("n_in,n_out,ncols", [(256, 5, 1), (4096, 64, 2), (12288, 36, 1), (1024, 16, 5), (2048, 8, 16)])
def test_gemv_vs_oracle(cuda, oracle, t, n_in, n_out, ncols):
    from rapier_b200 import ops

    w, xq = _case(oracle, t, n_in, n_out, ncols, n_in + n_out + t)
    y = empty_dev(ncols * n_out, torch.float32)
    ops.native_mmvq(t, to_dev(w), to_dev(xq), y, n_in, n_out, ncols)
    assert_close(to_np(y), oracle.mmvq(t, w, xq, n_in, n_out, ncols), what=f"kq gemv {t} {n_in}x{n_out}x{ncols}")


@pytest.mark.parametrize("t", [13, 12])
@pytest.mark.parametrize("ncols", [1, 3])
def test_isums_bit_exact(cuda, oracle, t, ncols):
    from rapier_b200 import ops

    n_in, n_out = 4096, 12
    w, xq = _case(oracle, t, n_in, n_out, ncols, 77 + t)
    out = empty_dev(ncols * n_out * 2 * (n_in // 32), torch.int32)
    ops.mmvq_isums(t, to_dev(w), to_dev(xq), out, n_in, n_out, ncols)
    assert np.array_equal(to_np(out), oracle.mmvq_isums(t, w, xq, n_in, n_out, ncols))


@pytest.mark.parametrize("t", [13, 12])
def test_res_epilogue(cuda, oracle, t):
    from rapier_b200 import ops

    n_in, n_out = 4096, 4096
    w, xq = _case(oracle, t, n_in, n_out, 1, 5 + t)
    res = oracle.synth_normal(3, n_out)
    want_y, want_p = oracle.mmvq_res(t, w, xq, res, n_in, n_out)
    y = to_dev(res.copy())  # y == res, as the reference calls it
    part = empty_dev(n_out // 4, torch.float32)
    (ops.native_q5_k_mmvq_res if t == 13 else ops.native_q4_k_mmvq_res)(to_dev(w), to_dev(xq), y, y, part, n_in, n_out)
    assert_close(to_np(y), want_y, what="kq res y")
    assert_close(to_np(part), want_p, what="kq res partials")


def test_argument_checks(cuda, oracle):
    from rapier_b200 import _lib, ops

    n_in, n_out = 512, 4
    w, xq = _case(oracle, 13, n_in, n_out, 1, 1)
    buf = torch.zeros(len(w) + 16, dtype=torch.uint8, device="cuda")
    buf[2:2 + len(w)] = to_dev(w)
    y = empty_dev(n_out, torch.float32)
    with pytest.raises(_lib.RkError) as ei:  # 2-byte aligned K-quant rows
        ops.native_mmvq(13, buf[2:], to_dev(xq), y, n_in, n_out, 1)
    assert ei.value.code == _lib.RK_EINVAL
    with pytest.raises(_lib.RkError) as ei:  # n_in not a multiple of 256
        ops.native_mmvq(13, to_dev(w), to_dev(xq), y, 480, n_out, 1)
    assert ei.value.code == _lib.RK_EINVAL
    with pytest.raises(_lib.RkError) as ei:  # no packed layout
        ops.mmvq_packed(13, to_dev(w), to_dev(xq), y, 1024, 4, 1)
    assert ei.value.code == _lib.RK_EUNSUPPORTED
