"""GPU parity of the norm / elementwise / Gated-DeltaNet / attention kernels against the CPU oracle,
through the C-ABI. Bit-exact (fp32 values and Q8_1 bytes) wherever the kernel reduces in the oracle's order:
exp, log1p and 1/sqrt are one exactly specified sequence on both sides (tests/test_math.py). Where the
C-ABI kernel sums in another order than the oracle restates (rk_rms_norm_rows, the split-L attention of
rk_gqa_decode_f16), fp32 outputs are compared within RTOL = 1e-3 (tests/_util.py) or tighter."""
import numpy as np
import pytest
import torch

from tests._util import assert_bits, assert_close, empty_dev, to_dev, to_np

pytestmark = pytest.mark.gpu
EPS = 1e-6


def _pos(p):
    return to_dev(np.array([p], np.int32))


def test_partials_and_add(cuda, oracle):
    from rapier_b200 import ops

    n = 4096
    x = oracle.synth_normal(1, n)
    o = oracle.synth_normal(2, n)
    dx, do = to_dev(x.copy()), to_dev(o)
    p = empty_dev(n // 4, torch.float32)
    ops.row_sum_partials(dx, p, n)
    assert np.array_equal(to_np(p), oracle.row_sumsq_partials(x))
    ops.add_partials(dx, do, p, n)
    wx, wp = oracle.add_partials(x, o)
    assert np.array_equal(to_np(dx), wx)
    assert np.array_equal(to_np(p), wp)


@pytest.mark.parametrize("ncols", [1, 2])
def test_rms_quant_and_norm_out(cuda, oracle, ncols):
    from rapier_b200 import ops

    cols = 4096
    x = oracle.synth_normal(3, cols * ncols)
    w = oracle.synth_normal(4, cols, std=0.02, mean=1.0)
    parts = np.concatenate([oracle.row_sumsq_partials(x[c * cols:(c + 1) * cols]) for c in range(ncols)])
    dx, dw, dp = to_dev(x), to_dev(w), to_dev(parts)
    y = empty_dev(ncols * cols // 32 * 36, torch.uint8)
    ops.rms_quant_apply(dx, dw, dp, y, cols, EPS, ncols=ncols)
    want = np.concatenate([oracle.rms_quant_q8_1(x[c * cols:(c + 1) * cols], w, parts[c * cols // 4:(c + 1) * cols // 4], EPS)
                           for c in range(ncols)])
    assert np.array_equal(to_np(y), want)
    out = empty_dev(ncols * cols, torch.float32)
    ops.rms_norm_out(dx, dw, dp, out, cols, EPS, ncols=ncols)
    wo = np.concatenate([oracle.rms_norm_out(x[c * cols:(c + 1) * cols], w, parts[c * cols // 4:(c + 1) * cols // 4], EPS)
                         for c in range(ncols)])
    assert_bits(to_np(out), wo, what="rms_norm_out")


def test_swiglu_sigmul_beta_gate(cuda, oracle):
    from rapier_b200 import ops

    n = 12288
    up, gate = oracle.synth_normal(5, n), oracle.synth_normal(6, n, std=2.0)
    y = empty_dev(n // 32 * 36, torch.uint8)
    ops.swiglu_quant(to_dev(up), to_dev(gate), y, n)
    assert np.array_equal(to_np(y), oracle.swiglu_q8_1(up, gate))
    y2 = empty_dev(n // 32 * 36, torch.uint8)
    ops.sig_mul_quant(to_dev(up), to_dev(gate), y2, n)
    assert np.array_equal(to_np(y2), oracle.sigmul_q8_1(up, gate))
    b, a = oracle.synth_normal(7, 32), oracle.synth_normal(8, 32)
    a[0] = 30.0  # softplus passthrough branch
    dt, ssm_a = oracle.synth_normal(9, 32, std=0.5), -np.exp(oracle.synth_normal(10, 32, std=0.5)).astype(np.float32)
    db, dg = to_dev(b.copy()), empty_dev(32, torch.float32)
    ops.beta_gate(db, to_dev(a), to_dev(dt), to_dev(ssm_a), dg, 32)
    wb, wg = oracle.beta_gate(b, a, dt, ssm_a)
    assert_bits(to_np(db), wb, what="beta")
    assert_bits(to_np(dg), wg, what="gate")


def test_rms_norm_rows_split_rope(cuda, oracle):
    from rapier_b200 import ops

    heads, hd = 16, 256
    qg = oracle.synth_normal(11, heads * 2 * hd)
    q, g = empty_dev(heads * hd, torch.float32), empty_dev(heads * hd, torch.float32)
    ops.split_qg(to_dev(qg), q, g, heads, hd)
    wq, wg = oracle.split_qg(qg, heads, hd)
    assert np.array_equal(to_np(q), wq) and np.array_equal(to_np(g), wg)
    w = oracle.synth_normal(12, hd, std=0.05, mean=1.0)
    ops.rms_norm_weighted(q, to_dev(w), heads, hd, EPS)
    wq = oracle.rms_norm_rows(wq, w, heads, hd, EPS)
    assert_close(to_np(q), wq, rtol=1e-5, what="rms rows")
    table = oracle.rope_table(1024, 64, 1e7)
    qn = to_np(q).copy()
    ops.rope_apply(q, heads, hd, 64, to_dev(table), 1024, _pos(777))
    assert np.array_equal(to_np(q), oracle.rope_apply(qn, heads, hd, 64, table, 777))
    # exactness of the rotation itself
    x = oracle.synth_normal(13, heads * hd)
    dx = to_dev(x)
    ops.rope_apply(dx, heads, hd, 64, to_dev(table), 1024, _pos(5))
    assert np.array_equal(to_np(dx), oracle.rope_apply(x, heads, hd, 64, table, 5))


def test_gdn_conv_l2(cuda, oracle):
    from rapier_b200 import ops

    C, qk_heads = 8192, 32
    ring = oracle.synth_normal(20, C * 4, std=0.5)
    conv_w = oracle.synth_normal(21, C * 4, std=0.3)
    pos = 10
    ring_g = to_dev(ring.copy())
    for step in range(3):  # three positions in a row: the ring rotates
        qkv = oracle.synth_normal(22 + step, C)
        h = empty_dev(C, torch.float32)
        ops.fused_gdn_conv_l2(ring_g, to_dev(qkv), to_dev(conv_w), h, C, qk_heads, EPS, _pos(pos + step))
        ring, want = oracle.gdn_conv_l2(ring, qkv, conv_w, C, qk_heads, EPS, pos + step)
        assert np.array_equal(to_np(ring_g), ring)
        assert_bits(to_np(h), want, what=f"conv_l2 step {step}")


def _gdn_inputs(oracle, seed, h_k=16, h_v=32):
    S = 128
    rng_seed = seed * 100
    state = oracle.synth_normal(rng_seed + 1, S * h_v * S, std=0.01)
    qk = oracle.synth_normal(rng_seed + 2, 2 * h_k * S)
    q = qk[:h_k * S].reshape(h_k, S)
    k = qk[h_k * S:].reshape(h_k, S)
    q = (q / np.linalg.norm(q, axis=1, keepdims=True)).astype(np.float32).ravel()
    k = (k / np.linalg.norm(k, axis=1, keepdims=True)).astype(np.float32).ravel()
    v = oracle.synth_normal(rng_seed + 3, h_v * S)
    gate = -np.abs(oracle.synth_normal(rng_seed + 4, h_v))
    beta = (1 / (1 + np.exp(-oracle.synth_normal(rng_seed + 5, h_v)))).astype(np.float32)
    z = oracle.synth_normal(rng_seed + 6, h_v * S)
    gamma = oracle.synth_normal(rng_seed + 7, S, std=0.1, mean=1.0)
    return state, q, k, v, gate.astype(np.float32), beta, z, gamma


def test_gdn_step_norm_silu_q8(cuda, oracle):
    from rapier_b200 import ops

    h_k, h_v = 16, 32
    state, q, k, v, gate, beta, z, gamma = _gdn_inputs(oracle, 1)
    ds = to_dev(state.copy())
    y = empty_dev(h_v * 128, torch.float32)
    q8 = empty_dev(h_v * 4 * 36, torch.uint8)
    ops.fused_gdn_step_norm_silu_q8(ds, to_dev(q), to_dev(k), to_dev(v), to_dev(gate), to_dev(beta), to_dev(z),
                                    to_dev(gamma), EPS, y, q8, h_k, h_v)
    ws, wy, wq8 = oracle.gdn_step_norm_silu_q8(state, q, k, v, gate, beta, z, gamma, EPS, h_k, h_v)
    assert_bits(to_np(ds), ws, what="state")
    assert_bits(to_np(y), wy, what="y")
    assert np.array_equal(to_np(q8), wq8)


def _fused_reference(oracle, proj, ring, conv_w, dt, ssm_a, gamma, state, h_k, h_v, pos, ncols):
    """The chain the fused kernel replaces: beta_gate -> conv_l2 -> step_norm_silu_q8, per column."""
    S = 128
    C = 2 * h_k * S + h_v * S
    ys, q8s, snap = [], [], None
    for c in range(ncols):
        col = proj[c]
        beta, g = oracle.beta_gate(col[C + h_v * S:C + h_v * S + h_v], col[C + h_v * S + h_v:], dt, ssm_a)
        ring, h = oracle.gdn_conv_l2(ring, col[:C], conv_w, C, 2 * h_k, EPS, pos + c)
        state, y, q8 = oracle.gdn_step_norm_silu_q8(state, h[:h_k * S], h[h_k * S:2 * h_k * S], h[2 * h_k * S:C], g,
                                                     beta, col[C:C + h_v * S], gamma, EPS, h_k, h_v)
        if c == 0:
            snap = state.copy()
        ys.append(y)
        q8s.append(q8)
    return ring, state, snap, np.concatenate(ys), np.concatenate(q8s)


@pytest.mark.parametrize("ncols", [1, 2])
def test_gdn_fused_vs_chain(cuda, oracle, ncols):
    from rapier_b200 import ops

    h_k, h_v, S = 16, 32, 128
    C = 2 * h_k * S + h_v * S
    stride = C + h_v * S + 2 * h_v
    proj = [oracle.synth_normal(40 + c, stride) for c in range(ncols)]
    state, *_ = _gdn_inputs(oracle, 2)
    ring = oracle.synth_normal(50, C * 4, std=0.5)
    conv_w = oracle.synth_normal(51, C * 4, std=0.3)
    dt = oracle.synth_normal(52, h_v, std=0.5)
    ssm_a = -np.exp(oracle.synth_normal(53, h_v, std=0.5)).astype(np.float32)
    gamma = oracle.synth_normal(54, S, std=0.1, mean=1.0)
    pos = 37
    d = dict(proj=to_dev(np.concatenate(proj)), ring=to_dev(ring.copy()), state=to_dev(state.copy()),
             snap=to_dev(np.zeros_like(state)), y=empty_dev(ncols * h_v * S, torch.float32),
             q8=empty_dev(ncols * h_v * 4 * 36, torch.uint8))
    ops.gdn_fused(d["proj"], stride, d["ring"], to_dev(conv_w), to_dev(dt), to_dev(ssm_a), to_dev(gamma), d["state"],
                  d["snap"], _pos(0), d["y"], d["q8"], h_k, h_v, ncols, _pos(pos), EPS)
    wring, wstate, wsnap, wy, wq8 = _fused_reference(oracle, proj, ring, conv_w, dt, ssm_a, gamma, state, h_k, h_v,
                                                     pos, ncols)
    assert np.array_equal(to_np(d["ring"]), wring)
    assert_bits(to_np(d["state"]), wstate, what="state")
    if ncols == 2:
        assert_bits(to_np(d["snap"]), wsnap, what="snapshot")
    assert_bits(to_np(d["y"]), wy, what="y")
    assert np.array_equal(to_np(d["q8"]), wq8)


def test_gdn_fused_two_tokens_bitwise_and_rollback(cuda, oracle):
    """A 2-token launch == two 1-token launches bit for bit (y, Q8_1, state), and a rollback launch reads
    the snapshot written after column 0."""
    from rapier_b200 import ops

    h_k, h_v, S = 16, 32, 128
    C = 2 * h_k * S + h_v * S
    stride = C + h_v * S + 2 * h_v
    proj = np.concatenate([oracle.synth_normal(60 + c, stride) for c in range(2)])
    state, *_ = _gdn_inputs(oracle, 3)
    ring = oracle.synth_normal(61, C * 4, std=0.5)
    conv_w, dt = to_dev(oracle.synth_normal(62, C * 4, std=0.3)), to_dev(oracle.synth_normal(63, h_v, std=0.5))
    ssm_a = to_dev(-np.exp(oracle.synth_normal(64, h_v, std=0.5)).astype(np.float32))
    gamma = to_dev(oracle.synth_normal(65, S, std=0.1, mean=1.0))
    pos = 100
    zero, one = _pos(0), _pos(1)

    def run(nc, col0_proj, st, rg, p, rollback, snap):
        y = empty_dev(nc * h_v * S, torch.float32)
        q8 = empty_dev(nc * h_v * 4 * 36, torch.uint8)
        ops.gdn_fused(col0_proj, stride, rg, conv_w, dt, ssm_a, gamma, st, snap, rollback, y, q8, h_k, h_v, nc,
                      _pos(p), EPS)
        return to_np(y), to_np(q8)

    dproj = to_dev(proj)
    # two single-token steps
    st1, rg1, sn1 = to_dev(state.copy()), to_dev(ring.copy()), to_dev(np.zeros_like(state))
    ya, qa = run(1, dproj, st1, rg1, pos, zero, sn1)
    after0 = to_np(st1).copy()
    yb, qb = run(1, dproj[stride:], st1, rg1, pos + 1, zero, sn1)
    # one 2-token step
    st2, rg2, sn2 = to_dev(state.copy()), to_dev(ring.copy()), to_dev(np.zeros_like(state))
    y2, q2 = run(2, dproj, st2, rg2, pos, zero, sn2)
    n = h_v * S
    assert np.array_equal(y2[:n].view(np.uint32), ya.view(np.uint32))
    assert np.array_equal(y2[n:].view(np.uint32), yb.view(np.uint32))
    assert np.array_equal(q2, np.concatenate([qa, qb]))
    assert np.array_equal(to_np(st2), to_np(st1))
    assert np.array_equal(to_np(sn2), after0)
    # reject: redo position pos+1 from the snapshot with rollback set; equals the single step from after0
    st3 = to_dev(after0.copy())
    rg3 = to_dev(to_np(rg2).copy())
    yc, _ = run(1, dproj[stride:], st2, rg2, pos + 1, one, sn2)
    yd, _ = run(1, dproj[stride:], st3, rg3, pos + 1, zero, to_dev(np.zeros_like(state)))
    assert np.array_equal(yc.view(np.uint32), yd.view(np.uint32))
    assert np.array_equal(to_np(st2), to_np(st3))


@pytest.mark.parametrize("L", [1, 300, 512, 8192, 65536])
@pytest.mark.parametrize("ncols", [1, 2])
def test_gqa_decode_vs_oracle(cuda, oracle, L, ncols):
    """The flash-decode GQA workload: 16 q heads, 4 kv heads, hd 256, fp16 KV ~ N(0, 1) at contexts up to 65536;
    column c attends 0..pos+c."""
    from rapier_b200 import ops

    n_head, n_kv, hd = 16, 4, 256
    max_ctx = L + 1
    pos = L - ncols  # last column sees exactly L tokens
    if pos < 0:
        pytest.skip("needs L >= ncols")
    rng = np.random.default_rng(L)
    k16 = rng.standard_normal((n_kv, max_ctx, hd)).astype(np.float16)
    v16 = rng.standard_normal((n_kv, max_ctx, hd)).astype(np.float16)
    q = (rng.standard_normal((ncols, n_head, hd)) * 0.5).astype(np.float32)
    dk, dv = to_dev(k16.view(np.uint16)), to_dev(v16.view(np.uint16))
    o = empty_dev(ncols * n_head * hd, torch.float32)
    sb = ops.gqa_scratch_bytes(n_head, ncols, max_ctx)
    scratch = empty_dev(sb // 4, torch.float32)
    ops.gqa_decode_f16(to_dev(q), dk, dv, o, n_head, n_kv, hd, ncols, _pos(pos), max_ctx, 0.0625, scratch, sb)
    got = to_np(o).reshape(ncols, n_head, hd)
    # oracle works on the reference's [ctx][n_kv][hd] layout
    kref = np.ascontiguousarray(k16.transpose(1, 0, 2)).view(np.uint16)
    vref = np.ascontiguousarray(v16.transpose(1, 0, 2)).view(np.uint16)
    for c in range(ncols):
        want = oracle.gqa_decode_f16(q[c].ravel(), kref.ravel(), vref.ravel(), n_head, n_kv, hd, pos + c + 1, 0.0625)
        assert_close(got[c].ravel(), want, what=f"gqa L={L} col {c}")
    if ncols == 2:  # column invariance: column 1 == a 1-column launch at pos+1
        o1 = empty_dev(n_head * hd, torch.float32)
        ops.gqa_decode_f16(to_dev(q[1]), dk, dv, o1, n_head, n_kv, hd, 1, _pos(pos + 1), max_ctx, 0.0625, scratch, sb)
        assert np.array_equal(to_np(o1).view(np.uint32), got[1].ravel().view(np.uint32))


def test_store_kv_and_bounds(cuda, oracle):
    from rapier_b200 import ops

    n_kv, hd, max_ctx = 4, 256, 64
    kc = torch.zeros(n_kv * max_ctx * hd, dtype=torch.int16, device="cuda")
    vc = torch.zeros_like(kc)
    k, v = oracle.synth_normal(70, n_kv * hd), oracle.synth_normal(71, n_kv * hd)
    ops.store_kv_f16(kc, vc, to_dev(k), to_dev(v), _pos(9), n_kv, hd, max_ctx)
    got = to_np(kc).view(np.uint16).reshape(n_kv, max_ctx, hd)
    assert np.array_equal(got[:, 9, :], oracle.f32_to_f16(k).reshape(n_kv, hd))
    assert np.count_nonzero(got[:, :9]) == 0
    assert ops.device_status() == 0
    # a position outside the cache is refused on the device: nothing is written, status bit 2 set
    ops.store_kv_f16(kc, vc, to_dev(k), to_dev(v), _pos(max_ctx), n_kv, hd, max_ctx)
    assert ops.device_status() & 4
    assert ops.device_status() == 0  # cleared


def test_argmax_ties_lowest_index(cuda, oracle):
    from rapier_b200 import ops

    n = 248320
    x = oracle.synth_normal(80, 2 * n)
    x[1000] = x[200000] = 50.0  # tie in column 0: lowest index wins
    x[n + 7] = np.nan
    x[n + 9] = 40.0
    out = empty_dev(2, torch.int32)
    ops.argmax(to_dev(x), n, 2, out)
    got = to_np(out)
    assert got[0] == 1000 == oracle.argmax(x[:n])
    assert got[1] == 9
