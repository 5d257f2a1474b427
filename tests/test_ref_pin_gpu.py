"""Pins the CPU oracle's Gated-DeltaNet restatement to the reference's own kernels: the reference's
src/fused_gdn.cu (conv + SiLU + L2 of fused_gdn.cu:113-133, the beta / gate projection of :135-162, the
delta-rule step + gated RMSNorm + Q8_1 of :39-111), compiled from the reference tree with this project's Q8_1
rule header into oracle/_ref/libref_gdn.so (oracle/Makefile, target `ref`), runs on the GPU, and the oracle
runs the same inputs on the CPU.

The reference kernels use the CUDA library's fast exp and 1/sqrt and a contracting compile, the oracle its
exactly specified sequences, so the two agree to float32 rounding, not bit for bit: states, outputs and
gates within 2e-5 of their scale (a few ulps after six chained steps); Q8_1 scales within one fp16 step and
codes within one, equal for at least 99 % of the values. The engine's kernels are in turn bitwise equal to
the oracle (test_kernels_gpu.py, test_engine_gpu.py), so these tests tie them to the reference's kernels."""
import ctypes as C
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "oracle", "_ref", "libref_gdn.so")
S = 128
H_K, H_V = 16, 32  # the 9B geometry's GDN heads
EPS = 1e-6
TOL = 2e-5


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(LIB):
        pytest.skip("oracle/_ref/libref_gdn.so not built (the reference tree was absent at build time)")
    lib = C.CDLL(LIB)
    P, F, I = C.c_void_p, C.c_float, C.c_int
    lib.ref_gdn_conv_l2.argtypes = [P, P, P, P, I, I, F, P]
    lib.ref_gdn_ab.argtypes = [P, P, P, P, P, P, P, I, I, P]
    lib.ref_gdn_step_norm_silu_q8.argtypes = [P, P, P, P, P, P, P, P, F, P, P, I, I, P]
    for f in (lib.ref_gdn_conv_l2, lib.ref_gdn_ab, lib.ref_gdn_step_norm_silu_q8):
        f.restype = None
    return lib


def _dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def _host(t):
    import torch

    torch.cuda.synchronize()
    return t.cpu().numpy()


def _stream():
    import torch

    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _close(got, want, what, tol=TOL):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    scale = max(float(np.max(np.abs(want))), 1e-30)
    err = float(np.max(np.abs(got - want))) / scale
    assert err <= tol, f"{what}: max |ref - oracle| = {err:.3g} of the scale"


def _q8_close(got, want, n_blocks, what):
    g, w = got.reshape(n_blocks, 36), want.reshape(n_blocks, 36)
    dg = g[:, 0:2].copy().view(np.float16).astype(np.float64).ravel()
    dw = w[:, 0:2].copy().view(np.float16).astype(np.float64).ravel()
    assert np.all(np.abs(dg - dw) <= np.spacing(np.abs(dw).astype(np.float16)).astype(np.float64)), what + ": d"
    cg, cw = g[:, 4:].view(np.int8).astype(np.int32), w[:, 4:].view(np.int8).astype(np.int32)
    assert np.max(np.abs(cg - cw)) <= 1, what + ": codes"
    assert np.mean(cg == cw) >= 0.99, what + ": codes"


def _unit_rows(rng, heads):
    x = rng.standard_normal((heads, S)).astype(np.float32)
    return (x / np.linalg.norm(x, axis=1, keepdims=True)).astype(np.float32).ravel()


def test_step_norm_silu_q8_matches_reference_kernel(cuda, oracle, ref):
    """fused_gdn_step_norm_silu_q8 (fused_gdn.cu:39-111, :211-216) against or_gdn_step_norm_silu_q8 over six
    chained steps of the 9B geometry's 32 v-heads (the modulo q/k pairing over 16 k-heads)."""
    import torch

    rng = np.random.default_rng(11)
    state = (rng.standard_normal(S * H_V * S) * 0.05).astype(np.float32)
    gamma = (1.0 + 0.1 * rng.standard_normal(S)).astype(np.float32)
    d_state = _dev(state)
    d_gamma = _dev(gamma)
    d_y = torch.empty(H_V * S, dtype=torch.float32, device="cuda")
    d_q8 = torch.empty(H_V * 4 * 36, dtype=torch.uint8, device="cuda")
    for step in range(6):
        q, k = _unit_rows(rng, H_K), _unit_rows(rng, H_K)
        v = rng.standard_normal(H_V * S).astype(np.float32)
        gate = rng.uniform(-3.0, -0.01, H_V).astype(np.float32)  # softplus(.) * ssm_a < 0: a decay
        beta = rng.uniform(0.05, 0.95, H_V).astype(np.float32)
        z = rng.standard_normal(H_V * S).astype(np.float32)
        dq, dk, dv, dg, db, dz = (_dev(a) for a in (q, k, v, gate, beta, z))
        ref.ref_gdn_step_norm_silu_q8(_ptr(d_state), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(dg), _ptr(db), _ptr(dz),
                                      _ptr(d_gamma), EPS, _ptr(d_y), _ptr(d_q8), H_K, H_V, _stream())
        state, y, q8 = oracle.gdn_step_norm_silu_q8(state, q, k, v, gate, beta, z, gamma, EPS, H_K, H_V)
        _close(_host(d_state), state, f"state after step {step}")
        _close(_host(d_y), y, f"y at step {step}")
        _q8_close(_host(d_q8), q8, H_V * 4, f"Q8_1 at step {step}")
        state = _host(d_state)  # continue both from the reference's state: each step is checked on its own


def test_conv_l2_matches_reference_kernel(cuda, oracle, ref):
    """fused_gdn_conv_l2 (fused_gdn.cu:113-133; a 3-deep shift register per channel) against
    or_gdn_conv_l2 (a 4-slot ring indexed by position) over five positions: the same causal window, SiLU and
    per-head L2 of the q and k heads."""
    channels = 2 * H_K * S + H_V * S
    qk_heads = 2 * H_K
    rng = np.random.default_rng(12)
    conv_w = (rng.standard_normal(channels * 4) * 0.5).astype(np.float32)
    d_hist = _dev(np.zeros(channels * 3, np.float32))
    d_w = _dev(conv_w)
    import torch

    d_h = torch.empty(channels, dtype=torch.float32, device="cuda")
    ring = np.zeros(channels * 4, np.float32)
    for pos in range(5):
        qkv = rng.standard_normal(channels).astype(np.float32)
        d_x = _dev(qkv)
        ref.ref_gdn_conv_l2(_ptr(d_hist), _ptr(d_x), _ptr(d_w), _ptr(d_h), channels, qk_heads, EPS, _stream())
        ring, h = oracle.gdn_conv_l2(ring, qkv, conv_w, channels, qk_heads, EPS, pos)
        got = _host(d_h)
        _close(got[: qk_heads * S], h[: qk_heads * S], f"q/k heads at position {pos}")
        _close(got[qk_heads * S:], h[qk_heads * S:], f"v channels at position {pos}")
        # the reference's register holds the last three inputs, oldest first: the ring's slots pos-2 .. pos
        hist = _host(d_hist).reshape(channels, 3)
        r = ring.reshape(channels, 4)
        want = np.stack([r[:, (pos - 2) & 3], r[:, (pos - 1) & 3], r[:, pos & 3]], axis=1)
        assert np.array_equal(hist, want), f"history at position {pos}"


def test_beta_gate_matches_reference_kernel(cuda, oracle, ref):
    """fused_gdn_ab (fused_gdn.cu:135-162: bf16 projections, then beta = sigmoid, gate = softplus(a + dt) *
    ssm_a with the passthrough above 20) against or_beta_gate on the same projections (computed here in
    float64 from the same bf16 weights), both branches of the softplus covered."""
    n_embd = 4096
    rng = np.random.default_rng(13)
    x = rng.standard_normal(n_embd).astype(np.float32)
    bf = lambda a: (a.astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)  # noqa: E731 (truncation)
    wa = bf(rng.standard_normal(H_V * n_embd) * 0.02)
    wb = bf(rng.standard_normal(H_V * n_embd) * 0.02)
    dt = rng.standard_normal(H_V).astype(np.float32)
    dt[:4] += 25.0  # a + dt above 20: softplus passes the value through
    ssm_a = (-np.exp(rng.standard_normal(H_V))).astype(np.float32)
    import torch

    d_gate = torch.empty(H_V, dtype=torch.float32, device="cuda")
    d_beta = torch.empty(H_V, dtype=torch.float32, device="cuda")
    dx, dwa, dwb, ddt, dsa = (_dev(a) for a in (x, wa, wb, dt, ssm_a))
    ref.ref_gdn_ab(_ptr(dx), _ptr(dwa), _ptr(dwb), _ptr(ddt), _ptr(dsa), _ptr(d_gate), _ptr(d_beta), n_embd, H_V,
                   _stream())
    f32 = lambda w: (w.astype(np.uint32) << 16).view(np.float32).astype(np.float64).reshape(H_V, n_embd)  # noqa: E731
    a_proj = (f32(wa) @ x.astype(np.float64)).astype(np.float32)
    b_proj = (f32(wb) @ x.astype(np.float64)).astype(np.float32)
    beta, gate = oracle.beta_gate(b_proj, a_proj, dt, ssm_a)
    assert np.any(a_proj[:4] + dt[:4] > 20.0) and np.any(a_proj + dt < 20.0)
    _close(_host(d_beta), beta, "beta", tol=1e-5)
    _close(_host(d_gate), gate, "gate", tol=1e-5)
