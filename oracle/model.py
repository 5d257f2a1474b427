"""CPU oracle of the whole decode step (TEST INFRASTRUCTURE ONLY): the reference's forward_token
(src/qwythos.cpp:1773-1824 -> launch_token_gpu :1228-1238 -> forward_gdn :1074-1149 / forward_attn
:1183-1226 / ffn :1011-1042) and its MTP draft (draft_predict :1316-1406, with the slot-0 seed
:2955-2958) restated over the oracle's per-kernel restatements (liboracle.so), on the synthetic model
the decode engine generates from the same seed: value(i) of tensor t = synth(hash(seed, t), i) * std +
mean, every matrix Q6_K-encoded by the restated encoder.

This module imports nothing from the product package: the geometry is a plain object (any object with
the `Config` fields works, e.g. the engine's own rk_model_config) and the tensor ids below are restated
constants (tests check them against the engine's).

The GEMVs run in the packed-tile kernel's fp32 summation order (oracle.mmvq_packed: the same integer
sums as the reference's lane order, oracle.mmvq, with a different fp32 rounding sequence) and attention
in the decode engine's flash-decode order (oracle.attn_flash_f16, chunk length by the engine's rule for
max_ctx), so the model's logits can be compared bit for bit; the reference-order restatements agree with
them within fp32 rounding (tests/test_oracle_golden.py).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import oracle as O

KS, KHD = 128, 256

# synthetic tensor ids: globals, and per-layer slots (layer il's tensor = 100 + 32 * il + slot; the MTP
# block is layer n_layer)
T_TOK_EMBD, T_OUT_NORM, T_OUTPUT, T_ENORM, T_HNORM, T_EH_PROJ, T_SHNORM = 1, 2, 3, 4, 5, 6, 7
L_ATTN_NORM, L_POST_NORM, L_FFN_UP, L_FFN_GATE, L_FFN_DOWN = 0, 1, 2, 3, 4
L_GDN_QKV, L_GDN_Z, L_GDN_BETA, L_GDN_ALPHA, L_GDN_OUT, L_GDN_CONV, L_GDN_A, L_GDN_DT, L_GDN_NORM = range(5, 14)
L_ATT_Q, L_ATT_K, L_ATT_V, L_ATT_O, L_ATT_QN, L_ATT_KN = range(5, 11)


def layer_tid(il: int, slot: int) -> int:
    return 100 + 32 * il + slot


@dataclass
class Config:
    """The hybrid model's geometry (the reference's compile-time constants, src/qwythos.cpp:33-44)."""
    n_layer: int = 32
    n_embd: int = 4096
    n_ff: int = 12288
    n_vocab: int = 248320
    ssm_h_k: int = 16
    ssm_h_v: int = 32
    n_head: int = 16
    n_head_kv: int = 4
    n_rot: int = 64
    attn_interval: int = 4
    has_mtp: int = 1
    max_ctx: int = 4096
    eps: float = 1e-6
    rope_base: float = 1e7
    seed: int = 1


def config_9b(max_ctx: int = 4096, seed: int = 1, n_layer: int = 32) -> Config:
    """Qwen3.5-9B / Qwythos-9B shapes."""
    return Config(n_layer=n_layer, max_ctx=max_ctx, seed=seed)


def config_tiny(max_ctx: int = 256, seed: int = 7, n_layer: int = 4, vocab: int = 4096) -> Config:
    """A small model with the same structure (GDN layers, attention every 4th layer, MTP block)."""
    return Config(n_layer=n_layer, n_embd=1024, n_ff=2048, n_vocab=vocab, ssm_h_k=4, ssm_h_v=8, n_head=4,
                  n_head_kv=1, max_ctx=max_ctx, seed=seed)


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
    def __init__(self, cfg, only_layers=None, with_embed=True, with_draft=None):
        """only_layers: generate just these layer indices (the others stay None); with_embed=False skips
        the token embedding (the CPU baseline times layers and the head only); with_draft (default
        cfg.has_mtp): build the MTP block (eh_proj, its attention layer, enorm / hnorm / shnorm)."""
        self.cfg = cfg
        s = int(cfg.seed)
        H, FF, V = cfg.n_embd, cfg.n_ff, cfg.n_vocab
        hk, hv, nh, nkv = cfg.ssm_h_k, cfg.ssm_h_v, cfg.n_head, cfg.n_head_kv
        self.H, self.FF, self.V, self.hk, self.hv, self.nh, self.nkv = H, FF, V, hk, hv, nh, nkv
        self.eps = np.float32(cfg.eps)
        self.max_ctx = int(cfg.max_ctx)
        self.chunk_len = O.attn_chunk_len(self.max_ctx)
        self.tok_embd = gen_q6k(s, T_TOK_EMBD, H, V) if with_embed else None
        self.out_norm = gen_f32(s, T_OUT_NORM, H, 0.02, 1.0)
        self.lm_head = gen_q6k(s, T_OUTPUT, H, V)
        self.C = 2 * hk * KS + hv * KS
        self.layers = []
        for il in range(cfg.n_layer):
            if only_layers is not None and il not in only_layers:
                self.layers.append(None)
                continue
            self.layers.append(self._layer(il, ((il + 1) % cfg.attn_interval) != 0))
        if with_draft is None:
            with_draft = bool(cfg.has_mtp)
        self.draft_layer = None
        if with_draft:
            self.enorm = gen_f32(s, T_ENORM, H, 0.02, 1.0)
            self.hnorm = gen_f32(s, T_HNORM, H, 0.02, 1.0)
            self.shnorm = gen_f32(s, T_SHNORM, H, 0.02, 1.0)
            self.eh_proj = gen_q6k(s, T_EH_PROJ, 2 * H, H)
            self.draft_layer = self._layer(cfg.n_layer, False)
        self.rope = O.rope_table(self.max_ctx, cfg.n_rot, cfg.rope_base)
        self.reset()

    def _layer(self, il: int, gdn: bool) -> dict:
        s = int(self.cfg.seed)
        H, FF, hk, hv, nh, nkv, C = self.H, self.FF, self.hk, self.hv, self.nh, self.nkv, self.C
        t = lambda slot: layer_tid(il, slot)  # noqa: E731
        L = {"gdn": gdn,
             "attn_norm": gen_f32(s, t(L_ATTN_NORM), H, 0.02, 1.0),
             "post_norm": gen_f32(s, t(L_POST_NORM), H, 0.02, 1.0),
             "upgate": np.concatenate([gen_q6k(s, t(L_FFN_UP), H, FF), gen_q6k(s, t(L_FFN_GATE), H, FF)]),
             "down": gen_q6k(s, t(L_FFN_DOWN), FF, H)}
        if gdn:
            L["in_proj"] = np.concatenate([gen_q6k(s, t(L_GDN_QKV), H, C), gen_q6k(s, t(L_GDN_Z), H, hv * KS),
                                           gen_q6k(s, t(L_GDN_BETA), H, hv), gen_q6k(s, t(L_GDN_ALPHA), H, hv)])
            L["out_proj"] = gen_q6k(s, t(L_GDN_OUT), hv * KS, H)
            L["conv_w"] = gen_f32(s, t(L_GDN_CONV), C * 4, 0.3, 0.0)
            L["ssm_a"] = gen_f32(s, t(L_GDN_A), hv, 0.5, 0.0, kind=1)
            L["dt"] = gen_f32(s, t(L_GDN_DT), hv, 0.5, 0.0)
            L["ssm_norm"] = gen_f32(s, t(L_GDN_NORM), KS, 0.02, 1.0)
        else:
            L["in_proj"] = np.concatenate([gen_q6k(s, t(L_ATT_Q), H, 2 * nh * KHD),
                                           gen_q6k(s, t(L_ATT_K), H, nkv * KHD),
                                           gen_q6k(s, t(L_ATT_V), H, nkv * KHD)])
            L["out_proj"] = gen_q6k(s, t(L_ATT_O), nh * KHD, H)
            L["q_norm"] = gen_f32(s, t(L_ATT_QN), KHD, 0.02, 1.0)
            L["k_norm"] = gen_f32(s, t(L_ATT_KN), KHD, 0.02, 1.0)
        return L

    def _kv(self):
        return {"k": np.zeros((self.max_ctx, self.nkv, KHD), np.uint16),
                "v": np.zeros((self.max_ctx, self.nkv, KHD), np.uint16)}

    def reset(self):
        self.state = {}
        for il, L in enumerate(self.layers):
            if L is None:
                continue
            if L["gdn"]:
                self.state[il] = {"ring": np.zeros(self.C * 4, np.float32),
                                  "ssm": np.zeros(KS * self.hv * KS, np.float32)}
            else:  # caches [ctx][n_kv][hd]
                self.state[il] = self._kv()
        self.draft_kv = self._kv() if self.draft_layer is not None else None
        # the final-normed hidden of the last forward() and its 4-row partials (the draft's h input)
        self.h = np.zeros(self.H, np.float32)
        self.hp = np.zeros(self.H // 4, np.float32)

    def fill(self, n_pos: int, seed: int = 1):
        """The decode engine's synthetic long context (rk_engine_session_fill): after reset, block li's
        (layer index, the MTP block last) seed sd = hash(seed, 1000 + li); K / V rows [0, n_pos) of every
        kv head = fp16 of N(0, 1) values from hash(sd, 1) / hash(sd, 2) (value index (head * n_pos + t) *
        256 + d); GDN states = N(0, 0.01) values from hash(sd, 3); conv rings zero."""
        self.reset()
        h64 = O.lib().or_hash64
        blocks = list(enumerate(self.layers))
        if self.draft_layer is not None:
            blocks.append((len(self.layers), self.draft_layer))
        for li, L in blocks:
            sd = int(h64(seed, 1000 + li))
            if L is None:
                continue
            st = self.draft_kv if li == len(self.layers) else self.state[li]
            if not L["gdn"]:
                for key, k in (("k", 1), ("v", 2)):
                    v = O.synth_normal(int(h64(sd, k)), self.nkv * n_pos * KHD, std=1.0)
                    st[key][:n_pos] = O.f32_to_f16(v.reshape(self.nkv, n_pos, KHD).transpose(1, 0, 2))
            else:
                st["ssm"] = O.synth_normal(int(h64(sd, 3)), KS * self.hv * KS, std=0.01)

    def embed(self, tok: int) -> np.ndarray:
        rb = self.H // 256 * 210
        return O.dequantize_weights(O.TYPE_Q6_K, self.tok_embd[tok * rb:(tok + 1) * rb], self.H, 1)

    def _attention(self, L, kv, x, xp, pos):
        """forward_attn (src/qwythos.cpp:1183-1226): attn_norm + Q8_1, q||k||v, attention, sig_mul + Q8_1,
        wo + residual."""
        H, nh, nkv, eps = self.H, self.nh, self.nkv, self.eps
        xq = O.rms_quant_q8_1(x, L["attn_norm"], xp, eps)
        rows = 2 * nh * KHD + 2 * nkv * KHD
        q3 = O.mmvq_packed(O.TYPE_Q6_K, L["in_proj"], xq, H, rows)
        _, oq = O.attn_flash_f16(q3, 1, rows, L["q_norm"], L["k_norm"], self.rope, self.cfg.n_rot, nh, nkv,
                                 kv["k"], kv["v"], pos, self.chunk_len, eps)
        return O.mmvq_packed(O.TYPE_Q6_K, L["out_proj"], oq, nh * KHD, H, res=x)

    def _ffn(self, L, x, xp):
        """ffn (src/qwythos.cpp:1011-1042): post_norm + Q8_1, up||gate, swiglu + Q8_1, down + residual."""
        H, FF = self.H, self.FF
        xq = O.rms_quant_q8_1(x, L["post_norm"], xp, self.eps)
        ug = O.mmvq_packed(O.TYPE_Q6_K, L["upgate"], xq, H, 2 * FF)
        sq = O.swiglu_q8_1(ug[:FF], ug[FF:])
        return O.mmvq_packed(O.TYPE_Q6_K, L["down"], sq, FF, H, res=x)

    def layer(self, il: int, x, xp, pos: int):
        """Trunk layer il (its mixer, then the FFN) on hidden x with partials xp at position pos; returns
        (x, xp) and updates the layer's state."""
        H, hk, hv, eps = self.H, self.hk, self.hv, self.eps
        Q6 = O.TYPE_Q6_K
        L, st = self.layers[il], self.state[il]
        if L["gdn"]:  # forward_gdn (src/qwythos.cpp:1074-1149)
            xq = O.rms_quant_q8_1(x, L["attn_norm"], xp, eps)
            rows = 2 * hk * KS + 2 * hv * KS + 2 * hv
            proj = O.mmvq_packed(Q6, L["in_proj"], xq, H, rows)
            C = self.C
            z = proj[C:C + hv * KS]
            beta, g = O.beta_gate(proj[C + hv * KS:C + hv * KS + hv], proj[C + hv * KS + hv:], L["dt"], L["ssm_a"])
            st["ring"], h = O.gdn_conv_l2(st["ring"], proj[:C], L["conv_w"], C, 2 * hk, eps, pos)
            st["ssm"], _, q8 = O.gdn_step_norm_silu_q8(st["ssm"], h[:hk * KS], h[hk * KS:2 * hk * KS],
                                                       h[2 * hk * KS:C], g, beta, z, L["ssm_norm"], eps, hk, hv)
            x, xp = O.mmvq_packed(Q6, L["out_proj"], q8, hv * KS, H, res=x)
        else:
            x, xp = self._attention(L, st, x, xp, pos)
        return self._ffn(L, x, xp)

    def head(self, x, xp):
        """Final norm + lm_head (src/qwythos.cpp:1234); keeps the final-normed hidden and its partials for
        the draft (:1236-1237)."""
        self.h = O.rms_norm_out(x, self.out_norm, xp, self.eps)
        self.hp = O.row_sumsq_partials(self.h)
        xq = O.rms_quant_q8_1(x, self.out_norm, xp, self.eps)
        return O.mmvq_packed(O.TYPE_Q6_K, self.lm_head, xq, self.H, self.V)

    def forward(self, tok: int, pos: int) -> np.ndarray:
        """One teacher-forced token: returns the logits (n_vocab) and updates the caches."""
        x = self.embed(tok)
        xp = O.row_sumsq_partials(x)
        for il in range(len(self.layers)):
            x, xp = self.layer(il, x, xp, pos)
        return self.head(x, xp)

    def draft(self, tok: int, pos: int, h=None, hp=None, with_head: bool = True):
        """draft_predict (src/qwythos.cpp:1316-1406) at draft position pos: eh = [enorm(emb(tok)) |
        hnorm(h)] (embedding half first, :1327-1332) -> Q8_1 -> eh_proj (2H -> H, no residual) -> the nextn
        attention layer with its own KV cache (slot pos) and FFN -> shared head norm -> lm_head. h / hp
        default to the last forward()'s final-normed hidden and partials; h = 0 seeds slot 0 (:2955-2958).
        Returns the draft logits, or None without the head (the cache-fill step)."""
        H, eps, D = self.H, self.eps, self.draft_layer
        Q6 = O.TYPE_Q6_K
        h = self.h if h is None else np.asarray(h, np.float32)
        hp = self.hp if hp is None else np.asarray(hp, np.float32)
        e = self.embed(tok)
        ep = O.row_sumsq_partials(e)
        eh = np.concatenate([O.rms_norm_out(e, self.enorm, ep, eps), O.rms_norm_out(h, self.hnorm, hp, eps)])
        ehq = O.quantize_q8_1(eh, 2 * H, 1)
        dx = O.mmvq_packed(Q6, self.eh_proj, ehq, 2 * H, H)
        dxp = O.row_sumsq_partials(dx)
        dx, dxp = self._attention(D, self.draft_kv, dx, dxp, pos)
        dx, dxp = self._ffn(D, dx, dxp)
        if not with_head:
            return None
        xq = O.rms_quant_q8_1(dx, self.shnorm, dxp, eps)
        return O.mmvq_packed(Q6, self.lm_head, xq, H, self.V)

    def generate(self, prompt, n_gen: int):
        """Greedy decoding (the reference's CLI loop without MTP, src/qwythos.cpp:2905-2952, :3184-3192):
        prompt positions teacher-forced, then n_gen argmax tokens."""
        self.reset()
        logits = None
        for p, t in enumerate(prompt):
            logits = self.forward(int(t), p)
        out = []
        pos = len(prompt)
        for _ in range(n_gen):
            tok = O.argmax(logits)
            out.append(tok)
            if len(out) == n_gen:
                break
            logits = self.forward(tok, pos)
            pos += 1
        return out
