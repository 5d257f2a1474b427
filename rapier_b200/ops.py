"""Host-side mirror of the reference's operator surface for the decode path.

The names, argument order and meaning follow strata::kernels as the reference engine calls them
(src/native_mmvq.cu:3054-3818, src/fused_gdn.cu:167-225 and the in-file kernels of src/qwythos.cpp),
so a port of the reference's own parity harness (src/test_res.cpp) reads the same. Buffers are CUDA
torch tensors or raw device pointers (int); `stream` is a torch.cuda.Stream, a raw cudaStream_t (int) or
None for torch's current stream.

Error behaviour mirrors the reference: a bad shape, pointer or stream raises ValueError (the reference
throws std::invalid_argument, src/native_mmvq.cu:2312-2331); a failed launch raises RuntimeError
(std::runtime_error, :2326-2331). The underlying RkError carries the RK_E* code.
"""
from __future__ import annotations

from . import _lib
from ._lib import RK_EINVAL, RK_EUNSUPPORTED, RkError, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K, TYPE_Q8_0

__all__ = [
    "TYPE_Q6_K", "TYPE_Q5_K", "TYPE_Q4_K", "TYPE_Q8_0", "RkError",
    "native_q8_1_bytes", "native_quantize_q8_1", "native_mmvq_weight_bytes", "native_mmvq",
    "native_q6_k_mmvq", "native_q8_0_mmvq", "native_q6_k_mmvq_res", "native_q8_0_mmvq_res",
    "native_q5_k_mmvq", "native_q4_k_mmvq", "native_q5_k_mmvq_res", "native_q4_k_mmvq_res",
    "packed_bytes", "pack_weights", "unpack_weights", "mmvq_packed", "mmvq_packed_ex", "mmvq_packed_res", "mmvq_isums",
    "row_sum_partials", "add_partials", "rms_quant_apply", "rms_norm_out", "swiglu_quant", "sig_mul_quant",
    "beta_gate", "rms_norm_weighted", "argmax", "fused_gdn_conv_l2", "fused_gdn_step_norm_silu_q8",
    "gdn_fused", "split_qg", "rope_apply", "store_kv_f16", "gqa_scratch_bytes", "gqa_decode_f16", "gqa_decode_f16_noalloc", "device_status",
]


class InvalidArgument(ValueError, RkError):
    """The reference's std::invalid_argument."""

    def __init__(self, code: int, func: str, msg: str):
        RkError.__init__(self, code, func, msg)


def _ptr(t) -> int:
    if t is None:
        return 0
    if isinstance(t, int):
        return t
    if hasattr(t, "data_ptr"):
        if not t.is_cuda:
            raise InvalidArgument(RK_EINVAL, "ops", "buffers must be CUDA tensors")
        return t.data_ptr()
    raise TypeError(f"expected a CUDA tensor or a device pointer, got {type(t)!r}")


def _stream(s) -> int:
    if s is None:
        import torch

        return torch.cuda.current_stream().cuda_stream
    if isinstance(s, int):
        return s
    return s.cuda_stream


def _call(name: str, *args) -> int:
    try:
        return _lib.call(name, *args)
    except RkError as e:
        if e.code in (RK_EINVAL, RK_EUNSUPPORTED):
            raise InvalidArgument(e.code, e.func, _lib.last_error()) from None
        raise


# ---- Q8_1 (src/native_mmvq.cu:3054-3071) ----
def native_q8_1_bytes(n_in: int, ncols: int) -> int:
    n = _lib.lib().rk_q8_1_bytes(n_in, ncols)
    if n == 0:
        raise InvalidArgument(RK_EINVAL, "rk_q8_1_bytes", "requires n_in > 0 divisible by 32 and ncols >= 1")
    return n


def native_quantize_q8_1(x, x_q8_1, n_in: int, ncols: int, stream=None) -> None:
    _call("rk_quantize_q8_1", _ptr(x), _ptr(x_q8_1), n_in, ncols, _stream(stream))


# ---- GGUF-layout GEMV (src/native_mmvq.cu:3187-3818) ----
def native_mmvq_weight_bytes(ggml_type: int, n_in: int, n_out: int) -> int:
    n = _lib.lib().rk_weight_bytes(ggml_type, n_in, n_out)
    if n == 0:
        raise InvalidArgument(RK_EINVAL, "rk_weight_bytes", "unsupported type or shape")
    return n


def native_mmvq(ggml_type: int, weights, x_q8_1, y, n_in: int, n_out: int, ncols: int, stream=None) -> None:
    _call("rk_mmvq", ggml_type, _ptr(weights), _ptr(x_q8_1), _ptr(y), n_in, n_out, ncols, _stream(stream))


def native_q6_k_mmvq(weights, x_q8_1, y, n_in, n_out, ncols, stream=None):
    native_mmvq(TYPE_Q6_K, weights, x_q8_1, y, n_in, n_out, ncols, stream)


def native_q8_0_mmvq(weights, x_q8_1, y, n_in, n_out, ncols, stream=None):
    native_mmvq(TYPE_Q8_0, weights, x_q8_1, y, n_in, n_out, ncols, stream)


def native_q6_k_mmvq_res(weights, x_q8_1, y, res, partials, n_in, n_out, stream=None):
    _call("rk_mmvq_res", TYPE_Q6_K, _ptr(weights), _ptr(x_q8_1), _ptr(y), _ptr(res), _ptr(partials), n_in, n_out,
          _stream(stream))


def native_q8_0_mmvq_res(weights, x_q8_1, y, res, partials, n_in, n_out, stream=None):
    _call("rk_mmvq_res", TYPE_Q8_0, _ptr(weights), _ptr(x_q8_1), _ptr(y), _ptr(res), _ptr(partials), n_in, n_out,
          _stream(stream))


def native_q5_k_mmvq(weights, x_q8_1, y, n_in, n_out, ncols, stream=None):
    native_mmvq(TYPE_Q5_K, weights, x_q8_1, y, n_in, n_out, ncols, stream)


def native_q4_k_mmvq(weights, x_q8_1, y, n_in, n_out, ncols, stream=None):
    native_mmvq(TYPE_Q4_K, weights, x_q8_1, y, n_in, n_out, ncols, stream)


def native_q5_k_mmvq_res(weights, x_q8_1, y, res, partials, n_in, n_out, stream=None):
    _call("rk_mmvq_res", TYPE_Q5_K, _ptr(weights), _ptr(x_q8_1), _ptr(y), _ptr(res), _ptr(partials), n_in, n_out,
          _stream(stream))


def native_q4_k_mmvq_res(weights, x_q8_1, y, res, partials, n_in, n_out, stream=None):
    _call("rk_mmvq_res", TYPE_Q4_K, _ptr(weights), _ptr(x_q8_1), _ptr(y), _ptr(res), _ptr(partials), n_in, n_out,
          _stream(stream))


# ---- packed-tile GEMV ----
def packed_bytes(ggml_type: int, n_in: int, n_out: int) -> int:
    return _lib.lib().rk_packed_bytes(ggml_type, n_in, n_out)


def pack_weights(ggml_type, src, dst, n_in, n_out, stream=None):
    _call("rk_pack_weights", ggml_type, _ptr(src), _ptr(dst), n_in, n_out, _stream(stream))


def unpack_weights(ggml_type, src, dst, n_in, n_out, stream=None):
    _call("rk_unpack_weights", ggml_type, _ptr(src), _ptr(dst), n_in, n_out, _stream(stream))


def mmvq_packed(ggml_type, packed, x_q8_1, y, n_in, n_out, ncols, stream=None):
    _call("rk_mmvq_packed", ggml_type, _ptr(packed), _ptr(x_q8_1), _ptr(y), n_in, n_out, ncols, _stream(stream))


def mmvq_packed_ex(ggml_type, packed, x_q8_1, y, n_in, n_out, ncols, flags, stream=None):
    _call("rk_mmvq_packed_ex", ggml_type, _ptr(packed), _ptr(x_q8_1), _ptr(y), n_in, n_out, ncols, flags,
          _stream(stream))


def mmvq_packed_res(ggml_type, packed, x_q8_1, y, res, partials, n_in, n_out, ncols, stream=None):
    _call("rk_mmvq_packed_res", ggml_type, _ptr(packed), _ptr(x_q8_1), _ptr(y), _ptr(res), _ptr(partials), n_in,
          n_out, ncols, _stream(stream))


def mmvq_isums(ggml_type, packed, x_q8_1, out, n_in, n_out, ncols, stream=None):
    _call("rk_mmvq_isums", ggml_type, _ptr(packed), _ptr(x_q8_1), _ptr(out), n_in, n_out, ncols, _stream(stream))


# ---- norms / elementwise (src/qwythos.cpp:602-715) ----
def row_sum_partials(x, partials, n, stream=None):
    _call("rk_row_sumsq_partials", _ptr(x), _ptr(partials), n, _stream(stream))


def add_partials(x, o, partials, n, stream=None):
    _call("rk_add_partials", _ptr(x), _ptr(o), _ptr(partials), n, _stream(stream))


def rms_quant_apply(x, w, partials, y, cols, eps, ncols=1, stream=None):
    _call("rk_rms_quant_q8_1", _ptr(x), _ptr(w), _ptr(partials), _ptr(y), cols, ncols, eps, _stream(stream))


def rms_norm_out(x, w, partials, out, cols, eps, ncols=1, stream=None):
    _call("rk_rms_norm_out", _ptr(x), _ptr(w), _ptr(partials), _ptr(out), cols, ncols, eps, _stream(stream))


def swiglu_quant(up, gate, y, n, stream=None):
    _call("rk_swiglu_q8_1", _ptr(up), _ptr(gate), _ptr(y), n, _stream(stream))


def sig_mul_quant(o, g, y, n, stream=None):
    _call("rk_sigmul_q8_1", _ptr(o), _ptr(g), _ptr(y), n, _stream(stream))


def beta_gate(beta, alpha, dt, ssm_a, gate, n, stream=None):
    _call("rk_beta_gate", _ptr(beta), _ptr(alpha), _ptr(dt), _ptr(ssm_a), _ptr(gate), n, _stream(stream))


def rms_norm_weighted(x, w, rows, cols, eps, stream=None):
    _call("rk_rms_norm_rows", _ptr(x), _ptr(w), rows, cols, eps, _stream(stream))


MATH_FNS = {"exp": 0, "log": 1, "log1p": 2, "sigmoid": 3, "silu": 4, "rsqrt": 5, "cuda_expf": 6}


def math_probe(fn: str, x, y, n, stream=None):
    """y = f(x) with the kernels' exactly specified fp32 sequence (rk_math_probe)."""
    _call("rk_math_probe", MATH_FNS[fn], _ptr(x), _ptr(y), n, _stream(stream))


def argmax(x, n, ncols, out, stream=None):
    _call("rk_argmax", _ptr(x), n, ncols, _ptr(out), _stream(stream))


# ---- Gated DeltaNet (src/fused_gdn.cu:167-225) ----
def fused_gdn_conv_l2(ring, qkv, conv_w, h, channels, qk_heads, eps, pos, stream=None):
    _call("rk_gdn_conv_l2", _ptr(ring), _ptr(qkv), _ptr(conv_w), _ptr(h), channels, qk_heads, eps, _ptr(pos),
          _stream(stream))


def fused_gdn_step_norm_silu_q8(state, q, k, v, gate, beta, z, gamma, eps, y, q8, h_k, h_v, stream=None):
    _call("rk_gdn_step_norm_silu_q8", _ptr(state), _ptr(q), _ptr(k), _ptr(v), _ptr(gate), _ptr(beta), _ptr(z),
          _ptr(gamma), eps, _ptr(y), _ptr(q8), h_k, h_v, _stream(stream))


def gdn_fused(proj, proj_stride, ring, conv_w, dt_bias, ssm_a, gamma, state, snap, rollback, y, q8, h_k, h_v, ncols,
              pos, eps, stream=None):
    _call("rk_gdn_fused", _ptr(proj), proj_stride, _ptr(ring), _ptr(conv_w), _ptr(dt_bias), _ptr(ssm_a), _ptr(gamma),
          _ptr(state), _ptr(snap), _ptr(rollback), _ptr(y), _ptr(q8), h_k, h_v, ncols, _ptr(pos), eps, _stream(stream))


# ---- attention (src/qwythos.cpp:320-442) ----
def split_qg(qg, q, g, heads, hd, stream=None):
    _call("rk_split_qg", _ptr(qg), _ptr(q), _ptr(g), heads, hd, _stream(stream))


def rope_apply(x, heads, hd, n_rot, table, max_pos, pos, stream=None):
    _call("rk_rope", _ptr(x), heads, hd, n_rot, _ptr(table), max_pos, _ptr(pos), _stream(stream))


def store_kv_f16(kcache, vcache, k, v, pos, n_kv, hd, max_ctx, stream=None):
    _call("rk_store_kv_f16", _ptr(kcache), _ptr(vcache), _ptr(k), _ptr(v), _ptr(pos), n_kv, hd, max_ctx,
          _stream(stream))


def gqa_scratch_bytes(n_head, ncols, max_ctx):
    return _lib.lib().rk_gqa_scratch_bytes(n_head, ncols, max_ctx)


def gqa_decode_f16(q, kcache, vcache, o, n_head, n_kv, hd, ncols, pos, max_ctx, scale, scratch, scratch_bytes,
                   stream=None):
    _call("rk_gqa_decode_f16", _ptr(q), _ptr(kcache), _ptr(vcache), _ptr(o), n_head, n_kv, hd, ncols, _ptr(pos),
          max_ctx, scale, _ptr(scratch), scratch_bytes, _stream(stream))


def gqa_decode_f16_noalloc(q, kcache, vcache, o, n_head, n_kv, hd, ncols, pos, max_ctx, scale, stream=None):
    """gqa_decode_f16 without a scratch buffer, for callers that cannot allocate device memory: the chunk
    partials use an array built into the library (16 MiB per device). Calls that overlap on the GPU race
    on that array; the first call on a device should come before any stream capture."""
    _call("rk_gqa_decode_f16_noalloc", _ptr(q), _ptr(kcache), _ptr(vcache), _ptr(o), n_head, n_kv, hd, ncols,
          _ptr(pos), max_ctx, scale, _stream(stream))


def device_status(clear: bool = True) -> int:
    return _lib.lib().rk_device_status(1 if clear else 0)
