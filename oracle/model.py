"""CPU oracle of the whole decode step (TEST INFRASTRUCTURE ONLY): the reference's forward_token
(src/qwythos.cpp:1773-1824 -> launch_token_gpu :1228-1238 -> forward_gdn :1074-1149 / forward_attn
:1183-1226 / ffn :1011-1042) restated over the oracle's per-kernel restatements (liboracle.so), on the
synthetic model the engine generates from the same seed (tensor ids and distributions as in
rapier_b200/csrc/engine.cu: value(i) = synth(hash(seed, tid), i) * std + mean; Q6_K by the shared encoder).

Meant for small configs (config_tiny); the 9B model is checked on the GPU by size-independent properties.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O

KS, KHD = 128, 256


def tensor_seed(seed: int, tid: int) -> int:
    return int(O.lib().or_hash64(seed, tid))


def gen_f32(seed: int, tid: int, n: int, std: float, mean: float, kind: int = 0) -> np.ndarray:
    v = O.synth_normal(tensor_seed(seed, tid), n, std=std, mean=mean)
    if kind == 1:  # ssm_a = -exp(value), in double
        v = (-np.exp(v.astype(np.float64))).astype(np.float32)
    return v


def gen_q6k(seed: int, tid: int, n_in: int, n_out: int) -> np.ndarray:
    w = O.synth_normal(tensor_seed(seed, tid), n_in * n_out, std=0.02)
    return O.quantize_weights(O.TYPE_Q6_K, w, n_in, n_out)


class Model:
    def __init__(self, cfg, only_layers=None, with_embed=True):
        """only_layers: generate just these layer indices (the others stay None); with_embed=False skips
        the token embedding (the CPU baseline times layers and the head only)."""
        from rapier_b200 import engine as E

        self.cfg = cfg
        s = cfg.seed
        H, FF, V = cfg.n_embd, cfg.n_ff, cfg.n_vocab
        hk, hv, nh, nkv = cfg.ssm_h_k, cfg.ssm_h_v, cfg.n_head, cfg.n_head_kv
        self.H, self.FF, self.V, self.hk, self.hv, self.nh, self.nkv = H, FF, V, hk, hv, nh, nkv
        self.eps = np.float32(cfg.eps)
        self.tok_embd = gen_q6k(s, E.T_TOK_EMBD, H, V) if with_embed else None
        self.out_norm = gen_f32(s, E.T_OUT_NORM, H, 0.02, 1.0)
        self.lm_head = gen_q6k(s, E.T_OUTPUT, H, V)
        self.layers = []
        C = 2 * hk * KS + hv * KS
        self.C = C
        for il in range(cfg.n_layer):
            if only_layers is not None and il not in only_layers:
                self.layers.append(None)
                continue
            t = lambda slot: E.layer_tid(il, slot)  # noqa: E731
            L = {"gdn": ((il + 1) % cfg.attn_interval) != 0,
                 "attn_norm": gen_f32(s, t(E.L_ATTN_NORM), H, 0.02, 1.0),
                 "post_norm": gen_f32(s, t(E.L_POST_NORM), H, 0.02, 1.0),
                 "upgate": np.concatenate([gen_q6k(s, t(E.L_FFN_UP), H, FF), gen_q6k(s, t(E.L_FFN_GATE), H, FF)]),
                 "down": gen_q6k(s, t(E.L_FFN_DOWN), FF, H)}
            if L["gdn"]:
                L["in_proj"] = np.concatenate([gen_q6k(s, t(E.L_GDN_QKV), H, C), gen_q6k(s, t(E.L_GDN_Z), H, hv * KS),
                                               gen_q6k(s, t(E.L_GDN_BETA), H, hv), gen_q6k(s, t(E.L_GDN_ALPHA), H, hv)])
                L["out_proj"] = gen_q6k(s, t(E.L_GDN_OUT), hv * KS, H)
                L["conv_w"] = gen_f32(s, t(E.L_GDN_CONV), C * 4, 0.3, 0.0)
                L["ssm_a"] = gen_f32(s, t(E.L_GDN_A), hv, 0.5, 0.0, kind=1)
                L["dt"] = gen_f32(s, t(E.L_GDN_DT), hv, 0.5, 0.0)
                L["ssm_norm"] = gen_f32(s, t(E.L_GDN_NORM), KS, 0.02, 1.0)
            else:
                L["in_proj"] = np.concatenate([gen_q6k(s, t(E.L_ATT_Q), H, 2 * nh * KHD),
                                               gen_q6k(s, t(E.L_ATT_K), H, nkv * KHD),
                                               gen_q6k(s, t(E.L_ATT_V), H, nkv * KHD)])
                L["out_proj"] = gen_q6k(s, t(E.L_ATT_O), nh * KHD, H)
                L["q_norm"] = gen_f32(s, t(E.L_ATT_QN), KHD, 0.02, 1.0)
                L["k_norm"] = gen_f32(s, t(E.L_ATT_KN), KHD, 0.02, 1.0)
            self.layers.append(L)
        self.rope = O.rope_table(cfg.max_ctx, cfg.n_rot, cfg.rope_base)
        self.reset()

    def reset(self):
        cfg = self.cfg
        self.state = {}
        for il, L in enumerate(self.layers):
            if L is None:
                continue
            if L["gdn"]:
                self.state[il] = {"ring": np.zeros(self.C * 4, np.float32),
                                  "ssm": np.zeros(KS * self.hv * KS, np.float32)}
            else:  # reference layout [ctx][n_kv][hd] for the oracle's attention
                self.state[il] = {"k": np.zeros((cfg.max_ctx, self.nkv, KHD), np.uint16),
                                  "v": np.zeros((cfg.max_ctx, self.nkv, KHD), np.uint16)}

    def embed(self, tok: int) -> np.ndarray:
        rb = self.H // 256 * 210
        return O.dequantize_weights(O.TYPE_Q6_K, self.tok_embd[tok * rb:(tok + 1) * rb], self.H, 1)

    def forward(self, tok: int, pos: int) -> np.ndarray:
        """One teacher-forced token: returns the logits (n_vocab) and updates the caches."""
        H, FF, hk, hv, nh, nkv, eps = self.H, self.FF, self.hk, self.hv, self.nh, self.nkv, self.eps
        Q6 = O.TYPE_Q6_K
        x = self.embed(tok)
        xp = O.row_sumsq_partials(x)
        for il, L in enumerate(self.layers):
            st = self.state[il]
            xq = O.rms_quant_q8_1(x, L["attn_norm"], xp, eps)
            if L["gdn"]:
                rows = 2 * hk * KS + 2 * hv * KS + 2 * hv
                proj = O.mmvq(Q6, L["in_proj"], xq, H, rows)
                C = self.C
                z = proj[C:C + hv * KS]
                beta, g = O.beta_gate(proj[C + hv * KS:C + hv * KS + hv], proj[C + hv * KS + hv:], L["dt"], L["ssm_a"])
                st["ring"], h = O.gdn_conv_l2(st["ring"], proj[:C], L["conv_w"], C, 2 * hk, eps, pos)
                st["ssm"], _, q8 = O.gdn_step_norm_silu_q8(st["ssm"], h[:hk * KS], h[hk * KS:2 * hk * KS],
                                                           h[2 * hk * KS:C], g, beta, z, L["ssm_norm"], eps, hk, hv)
                x, xp = O.mmvq_res(Q6, L["out_proj"], q8, x, hv * KS, H)
            else:
                rows = 2 * nh * KHD + 2 * nkv * KHD
                q3 = O.mmvq(Q6, L["in_proj"], xq, H, rows)
                q, gate = O.split_qg(q3[:2 * nh * KHD], nh, KHD)
                k = q3[2 * nh * KHD:2 * nh * KHD + nkv * KHD]
                v = q3[2 * nh * KHD + nkv * KHD:]
                q = O.rms_norm_rows(q, L["q_norm"], nh, KHD, eps)
                k = O.rms_norm_rows(k, L["k_norm"], nkv, KHD, eps)
                q = O.rope_apply(q, nh, KHD, self.cfg.n_rot, self.rope, pos)
                k = O.rope_apply(k, nkv, KHD, self.cfg.n_rot, self.rope, pos)
                st["k"][pos] = O.f32_to_f16(k).reshape(nkv, KHD)
                st["v"][pos] = O.f32_to_f16(v).reshape(nkv, KHD)
                o = O.gqa_decode_f16(q, st["k"].ravel(), st["v"].ravel(), nh, nkv, KHD, pos + 1, 0.0625)
                oq = O.sigmul_q8_1(o, gate)
                x, xp = O.mmvq_res(Q6, L["out_proj"], oq, x, nh * KHD, H)
            # ffn
            xq = O.rms_quant_q8_1(x, L["post_norm"], xp, eps)
            ug = O.mmvq(Q6, L["upgate"], xq, H, 2 * FF)
            sq = O.swiglu_q8_1(ug[:FF], ug[FF:])
            x, xp = O.mmvq_res(Q6, L["down"], sq, x, FF, H)
        xq = O.rms_quant_q8_1(x, self.out_norm, xp, eps)
        return O.mmvq(Q6, self.lm_head, xq, H, self.V)
