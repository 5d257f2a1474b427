"""ctypes bindings for the CPU oracle (oracle/liboracle.so). TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference leg load this module; the
product package (rapier_b200) never imports it. Every function takes and returns numpy arrays.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

TYPE_Q8_0 = 8
TYPE_Q4_K = 12
TYPE_Q5_K = 13
TYPE_Q6_K = 14

_lib = None


REF_TREE = "/root/reference"  # the reference checkout of the build container (absent on the GPU box)
REF_GDN_LIB = os.path.join(_HERE, "_ref", "libref_gdn.so")


def build() -> None:
    """Compile liboracle.so with the committed Makefile; where the reference tree is present, also the
    reference's own fused GDN kernels into _ref/libref_gdn.so (the GPU box only uses the prebuilt file)."""
    import subprocess

    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    if os.path.exists(os.path.join(REF_TREE, "src", "fused_gdn.cu")):
        subprocess.run(["make", "-s", "-C", _HERE, "ref", f"REF={REF_TREE}"], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = C.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i, _f, _d, _sz, _u64, _vp = C.c_int, C.c_float, C.c_double, C.c_size_t, C.c_uint64, C.c_void_p


def _declare(L):
    sig = {
        "or_f32_to_f16_n": (None, [_f32p, _u16p, _sz]),
        "or_f16_to_f32_n": (None, [_u16p, _f32p, _sz]),
        "or_hash64": (_u64, [_u64, _u64]),
        "or_synth_normal": (None, [_u64, _u64, _f, _f, _f32p, _sz]),
        "or_q8_1_bytes": (_sz, [_i, _i]),
        "or_quantize_q8_1": (None, [_f32p, _u8p, _i, _i]),
        "or_dequantize_q8_1": (None, [_u8p, _f32p, _i]),
        "or_weight_bytes": (_sz, [_i, _i, _i]),
        "or_dequant_kq": (None, [_i, _u8p, _f32p, _i]),
        "or_packed_bytes": (_sz, [_i, _i, _i]),
        "or_quantize_weights": (None, [_i, _f32p, _u8p, _i, _i]),
        "or_dequantize_weights": (None, [_i, _u8p, _f32p, _i, _i]),
        "or_pack_weights": (_i, [_i, _u8p, _u8p, _i, _i]),
        "or_unpack_weights": (_i, [_i, _u8p, _u8p, _i, _i]),
        "or_mmvq": (None, [_i, _u8p, _u8p, _f32p, _i, _i, _i]),
        "or_mmvq_res": (None, [_i, _u8p, _u8p, _f32p, _f32p, _f32p, _i, _i, _i]),
        "or_mmvq_packed": (None, [_i, _u8p, _u8p, _f32p, _vp, _vp, _i, _i, _i]),
        "or_mmvq_isums": (None, [_i, _u8p, _u8p, _i32p, _i, _i, _i]),
        "or_row_sumsq_partials": (None, [_f32p, _f32p, _i]),
        "or_add_partials": (None, [_f32p, _f32p, _f32p, _i]),
        "or_partials_sumsq": (_f, [_f32p, _i]),
        "or_rms_quant_q8_1": (None, [_f32p, _f32p, _f32p, _u8p, _i, _f]),
        "or_rms_norm_out": (None, [_f32p, _f32p, _f32p, _f32p, _i, _f]),
        "or_swiglu_q8_1": (None, [_f32p, _f32p, _u8p, _i]),
        "or_sigmul_q8_1": (None, [_f32p, _f32p, _u8p, _i]),
        "or_beta_gate": (None, [_f32p, _f32p, _f32p, _f32p, _f32p, _i]),
        "or_rms_norm_rows": (None, [_f32p, _f32p, _i, _i, _f]),
        "or_gdn_conv_l2": (None, [_f32p, _f32p, _f32p, _f32p, _i, _i, _f, _i]),
        "or_gdn_step_norm_silu_q8": (None, [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f,
                                            _f32p, _u8p, _i, _i]),
        "or_rope_table": (None, [_f32p, _i, _i, _d]),
        "or_rope_apply": (None, [_f32p, _i, _i, _i, _f32p, _i]),
        "or_split_qg": (None, [_f32p, _f32p, _f32p, _i, _i]),
        "or_store_kv_f16": (None, [_u16p, _u16p, _f32p, _f32p, _i, _i]),
        "or_gqa_decode_f16": (None, [_f32p, _u16p, _u16p, _f32p, _i, _i, _i, _i, _f]),
        "or_argmax": (_i, [_f32p, _i]),
        "or_math_n": (None, [_i, _f32p, _f32p, _sz]),
        "or_attn_flash_f16": (None, [_f32p, _i, _i, _f32p, _f32p, _f32p, _i, _i, _i, _u16p, _u16p, _i, _i, _f, _f,
                                     _f32p, _u8p]),
        "or_num_threads": (_i, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


# ---- fp16 ----
def f32_to_f16(x):
    x = _c(x, np.float32)
    y = np.empty(x.shape, np.uint16)
    lib().or_f32_to_f16_n(x.ravel(), y.ravel(), x.size)
    return y


def f16_to_f32(h):
    h = _c(h, np.uint16)
    y = np.empty(h.shape, np.float32)
    lib().or_f16_to_f32_n(h.ravel(), y.ravel(), h.size)
    return y


# ---- synthetic values ----
NORMAL_UNIT = float(np.float32(np.sqrt(3.0) / 65536.0))


def synth_scale(std: float) -> float:
    """The float32 multiplier that turns the centred sum of four u16 into a value of this std."""
    return float(np.float32(std * np.sqrt(3.0) / 65536.0))


def synth_normal(seed: int, n: int, std: float = 1.0, mean: float = 0.0, offset: int = 0):
    out = np.empty(n, np.float32)
    lib().or_synth_normal(seed, offset, synth_scale(std), mean, out, n)
    return out


# ---- Q8_1 ----
def quantize_q8_1(x, n_in: int, ncols: int = 1):
    x = _c(x, np.float32).ravel()
    assert x.size == n_in * ncols
    y = np.empty(lib().or_q8_1_bytes(n_in, ncols), np.uint8)
    lib().or_quantize_q8_1(x, y, n_in, ncols)
    return y


def dequantize_q8_1(y, n: int):
    x = np.empty(n, np.float32)
    lib().or_dequantize_q8_1(_c(y, np.uint8), x, n)
    return x


# ---- weights ----
def weight_bytes(t, n_in, n_out):
    return lib().or_weight_bytes(t, n_in, n_out)


def random_kquant_weights(t, n_in, n_out, seed):
    """Q5_K (13) / Q4_K (12) rows of random blocks: uniform code, scale and high-bit bytes, and the block
    scales d, dmin drawn as small positive fp16 (every byte pattern of the rest is a valid block)."""
    bb = 176 if t == TYPE_Q5_K else 144
    nb = n_out * (n_in // 256)
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    dm = np.stack([rng.uniform(0.5e-3, 2e-3, nb), rng.uniform(0.5e-3, 2e-3, nb)], 1).astype(np.float16)
    raw[:, 0:4] = dm.view(np.uint8).reshape(nb, 4)
    return raw.reshape(-1)


def dequant_kq(t, w, n_values):
    y = np.empty(n_values, np.float32)
    lib().or_dequant_kq(t, _c(w, np.uint8), y, n_values)
    return y


def quantize_weights(t, w, n_in, n_out):
    w = _c(w, np.float32).ravel()
    dst = np.empty(weight_bytes(t, n_in, n_out), np.uint8)
    lib().or_quantize_weights(t, w, dst, n_in, n_out)
    return dst


def dequantize_weights(t, w, n_in, n_out):
    out = np.empty(n_in * n_out, np.float32)
    lib().or_dequantize_weights(t, _c(w, np.uint8), out, n_in, n_out)
    return out


def pack_weights(t, raw, n_in, n_out):
    dst = np.empty(lib().or_packed_bytes(t, n_in, n_out), np.uint8)
    rc = lib().or_pack_weights(t, _c(raw, np.uint8), dst, n_in, n_out)
    if rc != 0:
        raise ValueError("pack_weights: unsupported shape")
    return dst


def unpack_weights(t, packed, n_in, n_out):
    dst = np.empty(weight_bytes(t, n_in, n_out), np.uint8)
    rc = lib().or_unpack_weights(t, _c(packed, np.uint8), dst, n_in, n_out)
    if rc != 0:
        raise ValueError("unpack_weights: unsupported shape")
    return dst


# ---- GEMV ----
def mmvq(t, w, xq, n_in, n_out, ncols=1):
    y = np.empty(n_out * ncols, np.float32)
    lib().or_mmvq(t, _c(w, np.uint8), _c(xq, np.uint8), y, n_in, n_out, ncols)
    return y


def mmvq_res(t, w, xq, res, n_in, n_out, ncols=1):
    y = np.empty(n_out * ncols, np.float32)
    nslots = (n_out + 3) // 4
    partials = np.empty(nslots * ncols, np.float32)
    lib().or_mmvq_res(t, _c(w, np.uint8), _c(xq, np.uint8), y, _c(res, np.float32), partials, n_in, n_out, ncols)
    return y, partials


def mmvq_packed(t, w, xq, n_in, n_out, ncols=1, res=None):
    """The GEMV in the packed-tile kernel's summation order (the decode engine's GEMVs): y, or with `res`
    (y = W x + res) the pair (y, 4-row partials)."""
    y = np.empty(ncols * n_out, np.float32)
    if res is None:
        lib().or_mmvq_packed(t, _c(w, np.uint8), _c(xq, np.uint8), y, None, None, n_in, n_out, ncols)
        return y
    res = _c(res, np.float32)
    p = np.empty(ncols * ((n_out + 3) // 4), np.float32)
    lib().or_mmvq_packed(t, _c(w, np.uint8), _c(xq, np.uint8), y, res.ctypes.data_as(C.c_void_p),
                         p.ctypes.data_as(C.c_void_p), n_in, n_out, ncols)
    return y, p


def mmvq_isums(t, w, xq, n_in, n_out, ncols=1):
    nsub = n_in // 16 if t == TYPE_Q6_K else (2 * (n_in // 32) if t in (TYPE_Q5_K, TYPE_Q4_K) else n_in // 32)
    out = np.empty(ncols * n_out * nsub, np.int32)
    lib().or_mmvq_isums(t, _c(w, np.uint8), _c(xq, np.uint8), out, n_in, n_out, ncols)
    return out


# ---- norms / elementwise ----
def row_sumsq_partials(x):
    x = _c(x, np.float32)
    p = np.empty((x.size + 3) // 4, np.float32)
    lib().or_row_sumsq_partials(x, p, x.size)
    return p


def add_partials(x, o):
    x = _c(x, np.float32).copy()
    p = np.empty((x.size + 3) // 4, np.float32)
    lib().or_add_partials(x, _c(o, np.float32), p, x.size)
    return x, p


def partials_sumsq(p):
    p = _c(p, np.float32)
    return lib().or_partials_sumsq(p, p.size)


def rms_quant_q8_1(x, w, partials, eps):
    x = _c(x, np.float32)
    y = np.empty(x.size // 32 * 36, np.uint8)
    lib().or_rms_quant_q8_1(x, _c(w, np.float32), _c(partials, np.float32), y, x.size, eps)
    return y


def rms_norm_out(x, w, partials, eps):
    x = _c(x, np.float32)
    out = np.empty_like(x)
    lib().or_rms_norm_out(x, _c(w, np.float32), _c(partials, np.float32), out, x.size, eps)
    return out


def swiglu_q8_1(up, gate):
    up = _c(up, np.float32)
    y = np.empty(up.size // 32 * 36, np.uint8)
    lib().or_swiglu_q8_1(up, _c(gate, np.float32), y, up.size)
    return y


def sigmul_q8_1(o, g):
    o = _c(o, np.float32)
    y = np.empty(o.size // 32 * 36, np.uint8)
    lib().or_sigmul_q8_1(o, _c(g, np.float32), y, o.size)
    return y


def beta_gate(beta, alpha, dt, ssm_a):
    beta = _c(beta, np.float32).copy()
    gate = np.empty_like(beta)
    lib().or_beta_gate(beta, _c(alpha, np.float32), _c(dt, np.float32), _c(ssm_a, np.float32), gate, beta.size)
    return beta, gate


def rms_norm_rows(x, w, rows, cols, eps):
    x = _c(x, np.float32).copy()
    lib().or_rms_norm_rows(x, _c(w, np.float32), rows, cols, eps)
    return x


# ---- GDN ----
def gdn_conv_l2(ring, qkv, conv_w, channels, qk_heads, eps, pos):
    ring = _c(ring, np.float32).copy()
    h = np.empty(channels, np.float32)
    lib().or_gdn_conv_l2(ring, _c(qkv, np.float32), _c(conv_w, np.float32), h, channels, qk_heads, eps, pos)
    return ring, h


def gdn_step_norm_silu_q8(state, q, k, v, gate, beta, z, gamma, eps, h_k, h_v):
    state = _c(state, np.float32).copy()
    y = np.empty(h_v * 128, np.float32)
    q8 = np.empty(h_v * 4 * 36, np.uint8)
    lib().or_gdn_step_norm_silu_q8(state, _c(q, np.float32), _c(k, np.float32), _c(v, np.float32),
                                   _c(gate, np.float32), _c(beta, np.float32), _c(z, np.float32),
                                   _c(gamma, np.float32), eps, y, q8, h_k, h_v)
    return state, y, q8


# ---- attention ----
def rope_table(max_pos, n_rot, freq_base):
    t = np.empty(max_pos * (n_rot // 2) * 2, np.float32)
    lib().or_rope_table(t, max_pos, n_rot, freq_base)
    return t


def rope_apply(x, heads, hd, n_rot, table, pos):
    x = _c(x, np.float32).copy()
    lib().or_rope_apply(x, heads, hd, n_rot, _c(table, np.float32), pos)
    return x


def split_qg(qg, heads, hd):
    q = np.empty(heads * hd, np.float32)
    g = np.empty(heads * hd, np.float32)
    lib().or_split_qg(_c(qg, np.float32), q, g, heads, hd)
    return q, g


def gqa_decode_f16(q, kc, vc, n_head, n_kv, hd, n_tok, scale):
    o = np.empty(n_head * hd, np.float32)
    lib().or_gqa_decode_f16(_c(q, np.float32), _c(kc, np.uint16), _c(vc, np.uint16), o, n_head, n_kv, hd, n_tok,
                            scale)
    return o


def attn_chunk_len(max_ctx: int) -> int:
    """Tokens per flash-decode chunk of a cache of max_ctx positions: the smallest of 32, 64, 128, 256 that
    splits the cache into at most 512 chunks (the decode engine's rule)."""
    n = 32
    while (max_ctx + n - 1) // n > 512 and n < 256:
        n *= 2
    return n


def attn_flash_f16(proj, ncols, proj_stride, qn, kn, rope, n_rot, n_head, n_kv, kc, vc, pos, chunk_len, eps,
                   scale=0.0625):
    """The attention step in the decode engine's flash-decode order (q/k norm, RoPE, fp16 K/V store at
    pos .. pos+ncols-1 into kc / vc [max_ctx][n_kv][256] in place, chunked softmax, combine). Returns
    (o [ncols][n_head][256], Q8_1 of o * sigmoid(gate) per column)."""
    assert kc.dtype == np.uint16 and kc.flags.c_contiguous and vc.dtype == np.uint16 and vc.flags.c_contiguous
    o = np.empty(ncols * n_head * 256, np.float32)
    q8 = np.empty(ncols * n_head * 8 * 36, np.uint8)
    lib().or_attn_flash_f16(_c(proj, np.float32), ncols, proj_stride, _c(qn, np.float32), _c(kn, np.float32),
                            _c(rope, np.float32), n_rot, n_head, n_kv, kc.reshape(-1), vc.reshape(-1), pos, chunk_len,
                            eps, scale, o, q8)
    return o, q8


def argmax(x):
    x = _c(x, np.float32)
    return lib().or_argmax(x, x.size)


def num_threads():
    return lib().or_num_threads()


# ---- exactly specified transcendentals (the sequences the CUDA kernels run) ----
MATH_FNS = {"exp": 0, "log": 1, "log1p": 2, "sigmoid": 3, "silu": 4, "rsqrt": 5}


def math(fn: str, x):
    x = _c(x, np.float32)
    y = np.empty_like(x)
    lib().or_math_n(MATH_FNS[fn], x.ravel(), y.ravel(), x.size)
    return y
