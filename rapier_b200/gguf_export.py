"""Write an engine's synthetic model as a qwen35 GGUF file (gguf-py), with the tensor names and metadata
keys the reference's loader reads (src/qwythos.cpp:1978-2124). rk_engine_create_gguf on the file gives an
engine with the same weights, so the loader can be checked end to end without a model download:

    from rapier_b200.engine import Engine, config_tiny
    from rapier_b200.gguf_export import export_gguf
    export_gguf(Engine(config_tiny()), "tiny.gguf")
"""
from __future__ import annotations

import numpy as np

from . import engine as E

COMMON = {E.L_ATTN_NORM: "attn_norm.weight", E.L_POST_NORM: "post_attention_norm.weight",
          E.L_FFN_UP: "ffn_up.weight", E.L_FFN_GATE: "ffn_gate.weight", E.L_FFN_DOWN: "ffn_down.weight"}
GDN = {E.L_GDN_QKV: "attn_qkv.weight", E.L_GDN_Z: "attn_gate.weight", E.L_GDN_BETA: "ssm_beta.weight",
       E.L_GDN_ALPHA: "ssm_alpha.weight", E.L_GDN_OUT: "ssm_out.weight", E.L_GDN_CONV: "ssm_conv1d.weight",
       E.L_GDN_A: "ssm_a", E.L_GDN_DT: "ssm_dt.bias", E.L_GDN_NORM: "ssm_norm.weight"}
ATT = {E.L_ATT_Q: "attn_q.weight", E.L_ATT_K: "attn_k.weight", E.L_ATT_V: "attn_v.weight",
       E.L_ATT_O: "attn_output.weight", E.L_ATT_QN: "attn_q_norm.weight", E.L_ATT_KN: "attn_k_norm.weight"}
QUANT = {E.L_FFN_UP, E.L_FFN_GATE, E.L_FFN_DOWN}  # per-layer Q6_K slots (plus the projections below)


def tensor_list(cfg):
    """(tensor id, GGUF name, quantized, (n_out, n_in) or (n,)) of every tensor of the model."""
    H, FF, V, S = cfg.n_embd, cfg.n_ff, cfg.n_vocab, 128
    hk, hv, nh, nkv = cfg.ssm_h_k, cfg.ssm_h_v, cfg.n_head, cfg.n_head_kv
    out = [(E.T_TOK_EMBD, "token_embd.weight", True, (V, H)), (E.T_OUT_NORM, "output_norm.weight", False, (H,)),
           (E.T_OUTPUT, "output.weight", True, (V, H))]
    for il in range(cfg.n_layer + (1 if cfg.has_mtp else 0)):
        gdn = il < cfg.n_layer and (il + 1) % cfg.attn_interval != 0
        b = f"blk.{il}."
        shapes = {E.L_ATTN_NORM: (H,), E.L_POST_NORM: (H,), E.L_FFN_UP: (FF, H), E.L_FFN_GATE: (FF, H),
                  E.L_FFN_DOWN: (H, FF)}
        if gdn:
            shapes.update({E.L_GDN_QKV: (2 * hk * S + hv * S, H), E.L_GDN_Z: (hv * S, H), E.L_GDN_BETA: (hv, H),
                           E.L_GDN_ALPHA: (hv, H), E.L_GDN_OUT: (H, hv * S), E.L_GDN_CONV: (2 * hk * S + hv * S, 4),
                           E.L_GDN_A: (hv,), E.L_GDN_DT: (hv,), E.L_GDN_NORM: (S,)})
            names = {**COMMON, **GDN}
            quant = QUANT | {E.L_GDN_QKV, E.L_GDN_Z, E.L_GDN_BETA, E.L_GDN_ALPHA, E.L_GDN_OUT}
        else:
            shapes.update({E.L_ATT_Q: (2 * nh * 256, H), E.L_ATT_K: (nkv * 256, H), E.L_ATT_V: (nkv * 256, H),
                           E.L_ATT_O: (H, nh * 256), E.L_ATT_QN: (256,), E.L_ATT_KN: (256,)})
            names = {**COMMON, **ATT}
            quant = QUANT | {E.L_ATT_Q, E.L_ATT_K, E.L_ATT_V, E.L_ATT_O}
        for slot, name in names.items():
            out.append((E.layer_tid(il, slot), b + name, slot in quant, shapes[slot]))
    if cfg.has_mtp:
        nx = f"blk.{cfg.n_layer}.nextn."
        out += [(E.T_EH_PROJ, nx + "eh_proj.weight", True, (H, 2 * H)), (E.T_ENORM, nx + "enorm.weight", False, (H,)),
                (E.T_HNORM, nx + "hnorm.weight", False, (H,)),
                (E.T_SHNORM, nx + "shared_head_norm.weight", False, (H,))]
    return out


def export_gguf(eng, path: str) -> None:
    import gguf

    cfg = eng.cfg
    w = gguf.GGUFWriter(path, "qwen35")
    w.add_uint32("qwen35.block_count", cfg.n_layer + (1 if cfg.has_mtp else 0))
    w.add_uint32("qwen35.nextn_predict_layers", 1 if cfg.has_mtp else 0)
    w.add_uint32("qwen35.full_attention_interval", cfg.attn_interval)
    w.add_uint32("qwen35.rope.dimension_count", cfg.n_rot)
    w.add_float64("qwen35.rope.freq_base", cfg.rope_base)
    w.add_float32("qwen35.attention.layer_norm_rms_epsilon", cfg.eps)
    for tid, name, quant, shape in tensor_list(cfg):
        raw = eng.read_tensor(tid)
        if quant:
            n_out, n_in = shape
            w.add_tensor(name, raw.reshape(n_out, n_in // 256 * 210), raw_dtype=gguf.GGMLQuantizationType.Q6_K)
        else:
            w.add_tensor(name, raw.view(np.float32).reshape(shape))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
