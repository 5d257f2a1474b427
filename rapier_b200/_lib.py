"""ctypes loader for librapier_b200.so and the raw rk_* C-ABI (include/rapier_b200.h).

The library must exist: there is no CPU fallback. Every wrapper raises RkError (with rk_last_error())
when an entry point returns a negative RK_E* code.
"""
from __future__ import annotations

import ctypes as C
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB_PATH = os.path.join(PKG, "librapier_b200.so")
HEADER = os.path.join(ROOT, "include", "rapier_b200.h")

RK_FLAG_STATIC_WEIGHTS = 1
RK_OK, RK_EINVAL, RK_ECUDA, RK_ENOMEM, RK_ERANGE, RK_EUNSUPPORTED = 0, -1, -2, -3, -4, -5
TYPE_Q8_0, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K = 8, 12, 13, 14
_CODE_NAMES = {RK_EINVAL: "RK_EINVAL", RK_ECUDA: "RK_ECUDA", RK_ENOMEM: "RK_ENOMEM", RK_ERANGE: "RK_ERANGE",
               RK_EUNSUPPORTED: "RK_EUNSUPPORTED"}


class RkError(RuntimeError):
    def __init__(self, code: int, func: str, msg: str):
        super().__init__(f"{func} -> {_CODE_NAMES.get(code, code)}: {msg}")
        self.code = code
        self.func = func


_lib = None

vp, i32, u32, f32, sz, i64 = C.c_void_p, C.c_int, C.c_uint, C.c_float, C.c_size_t, C.c_int64

class ModelConfig(C.Structure):
    """rk_model_config (include/rapier_b200.h)."""
    _fields_ = [("n_layer", C.c_int), ("n_embd", C.c_int), ("n_ff", C.c_int), ("n_vocab", C.c_int),
                ("ssm_h_k", C.c_int), ("ssm_h_v", C.c_int), ("n_head", C.c_int), ("n_head_kv", C.c_int),
                ("n_rot", C.c_int), ("attn_interval", C.c_int), ("has_mtp", C.c_int), ("max_ctx", C.c_int),
                ("eps", C.c_float), ("rope_base", C.c_double), ("seed", C.c_uint64),
                ("rope_yarn_factor", C.c_double), ("rope_orig_ctx", C.c_double)]


class GenStats(C.Structure):
    """rk_gen_stats (include/rapier_b200.h)."""
    _fields_ = [("prefill_ms", C.c_double), ("gen_ms", C.c_double), ("n_gen", C.c_int), ("mtp_steps", C.c_int),
                ("mtp_accepted", C.c_int), ("single_steps", C.c_int), ("graph_launches", C.c_int),
                ("kernels_per_single_step", C.c_int), ("kernels_per_round", C.c_int)]


class ProbeResult(C.Structure):
    """rk_probe_result (include/rapier_b200.h)."""
    _fields_ = [("ms", C.c_double), ("launches", C.c_int), ("weight_bytes", C.c_double), ("algo_bytes", C.c_double)]


# name -> (restype, argtypes); every function declared in include/rapier_b200.h appears here.
SIGNATURES = {
    "rk_last_error": (C.c_char_p, []),
    "rk_version": (i32, []),
    "rk_device_status": (u32, [i32]),
    "rk_q8_1_bytes": (sz, [i32, i32]),
    "rk_quantize_q8_1": (i32, [vp, vp, i32, i32, vp]),
    "rk_weight_bytes": (sz, [i32, i32, i32]),
    "rk_mmvq": (i32, [i32, vp, vp, vp, i32, i32, i32, vp]),
    "rk_mmvq_res": (i32, [i32, vp, vp, vp, vp, vp, i32, i32, vp]),
    "rk_packed_bytes": (sz, [i32, i32, i32]),
    "rk_pack_weights": (i32, [i32, vp, vp, i32, i32, vp]),
    "rk_unpack_weights": (i32, [i32, vp, vp, i32, i32, vp]),
    "rk_mmvq_packed": (i32, [i32, vp, vp, vp, i32, i32, i32, vp]),
    "rk_mmvq_packed_ex": (i32, [i32, vp, vp, vp, i32, i32, i32, u32, vp]),
    "rk_mmvq_packed_res": (i32, [i32, vp, vp, vp, vp, vp, i32, i32, i32, vp]),
    "rk_mmvq_isums": (i32, [i32, vp, vp, vp, i32, i32, i32, vp]),
    "rk_row_sumsq_partials": (i32, [vp, vp, i32, vp]),
    "rk_add_partials": (i32, [vp, vp, vp, i32, vp]),
    "rk_rms_quant_q8_1": (i32, [vp, vp, vp, vp, i32, i32, f32, vp]),
    "rk_rms_norm_out": (i32, [vp, vp, vp, vp, i32, i32, f32, vp]),
    "rk_swiglu_q8_1": (i32, [vp, vp, vp, i32, vp]),
    "rk_sigmul_q8_1": (i32, [vp, vp, vp, i32, vp]),
    "rk_beta_gate": (i32, [vp, vp, vp, vp, vp, i32, vp]),
    "rk_rms_norm_rows": (i32, [vp, vp, i32, i32, f32, vp]),
    "rk_argmax": (i32, [vp, i32, i32, vp, vp]),
    "rk_math_probe": (i32, [i32, vp, vp, i32, vp]),
    "rk_gdn_conv_l2": (i32, [vp, vp, vp, vp, i32, i32, f32, vp, vp]),
    "rk_gdn_step_norm_silu_q8": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, f32, vp, vp, i32, i32, vp]),
    "rk_split_qg": (i32, [vp, vp, vp, i32, i32, vp]),
    "rk_gdn_fused": (i32, [vp, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, vp, f32, vp]),
    "rk_rope": (i32, [vp, i32, i32, i32, vp, i32, vp, vp]),
    "rk_store_kv_f16": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, vp]),
    "rk_gqa_scratch_bytes": (sz, [i32, i32, i32]),
    "rk_gqa_decode_f16": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, vp, i32, f32, vp, sz, vp]),
    "rk_gqa_decode_f16_noalloc": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, vp, i32, f32, vp]),
    "rk_model_config_9b": (None, [C.POINTER(ModelConfig), i32, C.c_uint64]),
    "rk_engine_create": (i32, [C.POINTER(ModelConfig), i32, C.POINTER(vp)]),
    "rk_engine_destroy": (i32, [vp]),
    "rk_engine_reset": (i32, [vp]),
    "rk_engine_generate": (i32, [vp, C.POINTER(C.c_int), i32, i32, i32, C.POINTER(C.c_int), C.POINTER(GenStats)]),
    "rk_engine_step": (i32, [vp, C.POINTER(C.c_int), i32, i32, vp, C.POINTER(C.c_int)]),
    "rk_engine_draft_step": (i32, [vp, i32, i32, i32, vp, C.POINTER(C.c_int)]),
    "rk_engine_force_candidates": (i32, [vp, C.POINTER(C.c_int), i32]),
    "rk_engine_session_reset": (i32, [vp]),
    "rk_engine_session_run": (i32, [vp, C.POINTER(C.c_int), i32, i32, i32, i32, C.POINTER(C.c_int),
                                    C.POINTER(C.c_int), vp, C.POINTER(GenStats)]),
    "rk_engine_session_pos": (i32, [vp]),
    "rk_engine_session_fill": (i32, [vp, i32, C.c_uint64]),
    "rk_engine_read_tensor": (sz, [vp, i32, vp, sz]),
    "rk_engine_device_bytes": (sz, [vp]),
    "rk_engine_mode": (i32, [vp]),
    "rk_gguf_model_config": (i32, [C.c_char_p, i32, C.POINTER(ModelConfig)]),
    "rk_engine_create_gguf": (i32, [C.c_char_p, i32, i32, i32, i32, C.POINTER(vp)]),
    "rk_rope_table": (i32, [i32, C.c_double, C.c_double, C.c_double, i32, vp]),
    "rk_engine_create_tp": (i32, [C.POINTER(ModelConfig), i32, i32, i32, C.POINTER(vp)]),
    "rk_tp_handle_bytes": (sz, []),
    "rk_engine_tp_export": (i32, [vp, vp, sz]),
    "rk_engine_tp_connect": (i32, [vp, vp, sz]),
    "rk_engine_tp_resync": (i32, [vp]),
    "rk_engine_trace": (i32, [vp, i32, C.POINTER(C.c_double), C.POINTER(C.c_int), i32, C.POINTER(C.c_double), i32]),
    "rk_engine_probe_gemv": (i32, [vp, i32, i32, C.POINTER(ProbeResult)]),
}


def header_functions() -> list[str]:
    """Names of every function the public header declares."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(rk_[a-z0-9_]+)\s*\(", text)))


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m rapier_b200.build` "
                              "(there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().rk_last_error().decode()


def call(name: str, *args) -> int:
    """Call an int-returning entry point; raise RkError on a negative code."""
    rc = getattr(lib(), name)(*args)
    if rc < 0:
        raise RkError(rc, name, last_error())
    return rc
