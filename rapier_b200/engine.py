"""Python wrapper over the C++ decode engine (rk_engine_* in include/rapier_b200.h).

    from rapier_b200.engine import Engine, config_9b
    eng = Engine(config_9b(max_ctx=512, seed=1))
    ids, stats = eng.generate(prompt, n_gen=400, mtp=True)
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import GenStats, ModelConfig, ProbeResult, RkError

# synthetic tensor ids (engine.cu): globals and per-layer slots, layer il's tensor = 100 + 32*il + slot
T_TOK_EMBD, T_OUT_NORM, T_OUTPUT, T_ENORM, T_HNORM, T_EH_PROJ, T_SHNORM = 1, 2, 3, 4, 5, 6, 7
L_ATTN_NORM, L_POST_NORM, L_FFN_UP, L_FFN_GATE, L_FFN_DOWN = 0, 1, 2, 3, 4
L_GDN_QKV, L_GDN_Z, L_GDN_BETA, L_GDN_ALPHA, L_GDN_OUT, L_GDN_CONV, L_GDN_A, L_GDN_DT, L_GDN_NORM = 5, 6, 7, 8, 9, 10, 11, 12, 13
L_ATT_Q, L_ATT_K, L_ATT_V, L_ATT_O, L_ATT_QN, L_ATT_KN = 5, 6, 7, 8, 9, 10


def layer_tid(il: int, slot: int) -> int:
    return 100 + 32 * il + slot


def config_9b(max_ctx: int = 4096, seed: int = 1) -> ModelConfig:
    c = ModelConfig()
    _lib.lib().rk_model_config_9b(C.byref(c), max_ctx, seed)
    return c


def config_tiny(max_ctx: int = 256, seed: int = 7, n_layer: int = 4, vocab: int = 4096) -> ModelConfig:
    """A small model with the same structure (GDN layers and an attention layer every 4th, MTP block)."""
    c = config_9b(max_ctx, seed)
    c.n_layer, c.n_embd, c.n_ff, c.n_vocab = n_layer, 1024, 2048, vocab
    c.ssm_h_k, c.ssm_h_v, c.n_head, c.n_head_kv = 4, 8, 4, 1
    return c


def gguf_config(path: str, max_ctx: int = 4096) -> ModelConfig:
    """The model geometry of a qwen35 GGUF file (rk_gguf_model_config; reads the file only)."""
    c = ModelConfig()
    _lib.call("rk_gguf_model_config", str(path).encode(), max_ctx, C.byref(c))
    return c


class _engine_mode:
    """Sets RK_ENGINE_MODE around an engine's creation (the library reads it there)."""

    def __init__(self, mode):
        self.mode = mode

    def __enter__(self):
        import os

        self.old = os.environ.get("RK_ENGINE_MODE")
        if self.mode is not None:
            os.environ["RK_ENGINE_MODE"] = self.mode

    def __exit__(self, *exc):
        import os

        if self.mode is not None:
            if self.old is None:
                os.environ.pop("RK_ENGINE_MODE", None)
            else:
                os.environ["RK_ENGINE_MODE"] = self.old


class Engine:
    """mode: None (the library default, RK_ENGINE_MODE or graph), "persistent" or "graph"; the executor is
    chosen when the engine is created (the library reads RK_ENGINE_MODE then). tp_rank / tp_size: this process's shard
    under tensor parallelism (rk_engine_create_tp); connect the ranks with connect_tp() before use."""

    def __init__(self, cfg: ModelConfig, device: int = 0, mode: str | None = None, tp_rank: int = 0,
                 tp_size: int = 1, _gguf: str | None = None):
        self.cfg = cfg
        self.tp_rank, self.tp_size = tp_rank, tp_size
        h = C.c_void_p()
        with _engine_mode(mode):
            if _gguf is None:
                _lib.call("rk_engine_create_tp", C.byref(cfg), device, tp_rank, tp_size, C.byref(h))
            else:
                _lib.call("rk_engine_create_gguf", _gguf.encode(), device, cfg.max_ctx, tp_rank, tp_size,
                          C.byref(h))
        self._h = h

    @classmethod
    def from_gguf(cls, path: str, device: int = 0, max_ctx: int = 4096, mode: str | None = None,
                  tp_rank: int = 0, tp_size: int = 1) -> "Engine":
        """An engine over the weights of a qwen35 GGUF file (Q6_K matrices; rk_engine_create_gguf)."""
        return cls(gguf_config(path, max_ctx), device, mode, tp_rank, tp_size, _gguf=str(path))

    def close(self):
        if self._h:
            _lib.lib().rk_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        _lib.call("rk_engine_reset", self._h)

    def generate(self, prompt, n_gen: int, mtp: bool = False):
        p = (C.c_int * len(prompt))(*[int(t) for t in prompt])
        out = (C.c_int * n_gen)()
        st = GenStats()
        _lib.call("rk_engine_generate", self._h, p, len(prompt), n_gen, 1 if mtp else 0, out, C.byref(st))
        stats = {f: getattr(st, f) for f, _ in GenStats._fields_}
        return np.frombuffer(out, dtype=np.int32).copy(), stats

    # ---- serving session (rk_engine_session_*; the reference's --serve loop) ----
    def session_reset(self):
        _lib.call("rk_engine_session_reset", self._h)

    def session_run(self, tokens, n_gen: int, mtp: bool = False, eos: int = -1, first_logits: bool = False):
        """Ingest the pending token and `tokens`, generate up to n_gen tokens (stop after `eos`). Returns
        (ids, stats, logits of the first generated token or None)."""
        n = len(tokens)
        t = (C.c_int * max(1, n))(*[int(x) for x in tokens])
        out = (C.c_int * n_gen)()
        n_out = C.c_int(0)
        st = GenStats()
        lg = np.empty(self.cfg.n_vocab // self.tp_size, np.float32) if first_logits else None
        _lib.call("rk_engine_session_run", self._h, t, n, n_gen, 1 if mtp else 0, eos, out, C.byref(n_out),
                  lg.ctypes.data_as(C.c_void_p) if first_logits else None, C.byref(st))
        stats = {f: getattr(st, f) for f, _ in GenStats._fields_}
        return np.frombuffer(out, dtype=np.int32)[:n_out.value].copy(), stats, lg

    def session_fill(self, n_pos: int, seed: int = 1):
        """A synthetic context of n_pos tokens (rk_engine_session_fill): seeded caches, session after them."""
        _lib.call("rk_engine_session_fill", self._h, n_pos, seed)

    @property
    def session_pos(self) -> int:
        return _lib.lib().rk_engine_session_pos(self._h)

    def tp_export(self) -> bytes:
        """This rank's exchange-memory handle (rk_engine_tp_export)."""
        n = _lib.lib().rk_tp_handle_bytes()
        buf = (C.c_uint8 * n)()
        _lib.call("rk_engine_tp_export", self._h, buf, n)
        return bytes(buf)

    def tp_connect(self, handles: list) -> None:
        """Map every rank's exchange memory (handles in rank order, rk_engine_tp_connect)."""
        n = _lib.lib().rk_tp_handle_bytes()
        blob = b"".join(bytes(hh) for hh in handles)
        if len(blob) != n * self.tp_size:
            raise ValueError("one handle per rank expected")
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        _lib.call("rk_engine_tp_connect", self._h, buf, n)

    def tp_resync(self) -> None:
        """After a failed tensor-parallel call: clear this rank's exchange epochs and flags
        (rk_engine_tp_resync). Call on every rank with no kernel running, meet on the host, then reset."""
        _lib.call("rk_engine_tp_resync", self._h)

    def connect_tp(self, group=None) -> None:
        """Exchange the handles over torch.distributed (any backend; `group` spans this engine's ranks, in
        tensor-parallel rank order) and connect."""
        import torch
        import torch.distributed as dist

        mine = self.tp_export()
        dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
        t = torch.tensor(list(mine), dtype=torch.uint8, device=dev)
        got = [torch.empty_like(t) for _ in range(self.tp_size)]
        dist.all_gather(got, t, group=group)
        self.tp_connect([bytes(g.cpu().tolist()) for g in got])

    def step(self, tokens, pos: int, want_logits: bool = True):
        n = len(tokens)
        t = (C.c_int * n)(*[int(x) for x in tokens])
        am = (C.c_int * n)()
        logits = np.empty(n * (self.cfg.n_vocab // self.tp_size), np.float32) if want_logits else None
        _lib.call("rk_engine_step", self._h, t, n, pos,
                  logits.ctypes.data_as(C.c_void_p) if want_logits else None, am)
        return (logits.reshape(n, -1) if want_logits else None), list(am)

    def draft_step(self, tok: int, pos: int, h_zero: bool = False, want_logits: bool = True):
        """The MTP draft alone at draft position pos on (emb(tok), the last trunk pass's normed hidden, or 0)
        (rk_engine_draft_step). Returns (logits or None, argmax id)."""
        logits = np.empty(self.cfg.n_vocab // self.tp_size, np.float32) if want_logits else None
        am = C.c_int(0)
        _lib.call("rk_engine_draft_step", self._h, int(tok), int(pos), 1 if h_zero else 0,
                  logits.ctypes.data_as(C.c_void_p) if want_logits else None, C.byref(am))
        return logits, am.value

    def force_candidates(self, tokens_by_pos=None):
        """Forced MTP draft candidates by position (rk_engine_force_candidates; -1 keeps the draft's own);
        None clears them."""
        toks = [] if tokens_by_pos is None else [int(t) for t in tokens_by_pos]
        arr = (C.c_int * max(1, len(toks)))(*toks)
        _lib.call("rk_engine_force_candidates", self._h, arr, len(toks))

    def read_tensor(self, tid: int) -> np.ndarray:
        L = _lib.lib()
        n = L.rk_engine_read_tensor(self._h, tid, None, 0)
        if n == 0:
            raise RkError(_lib.RK_EINVAL, "rk_engine_read_tensor", f"no tensor {tid}")
        buf = np.empty(n, np.uint8)
        got = L.rk_engine_read_tensor(self._h, tid, buf.ctypes.data_as(C.c_void_p), n)
        if got != n:
            raise RkError(_lib.RK_ECUDA, "rk_engine_read_tensor", "copy failed")
        return buf

    def probe_gemv(self, ncols: int = 1, iters: int = 10) -> dict:
        r = ProbeResult()
        _lib.call("rk_engine_probe_gemv", self._h, ncols, iters, C.byref(r))
        return {"ms": r.ms, "iters": iters, "launches": r.launches, "weight_bytes": r.weight_bytes,
                "algo_bytes": r.algo_bytes}

    def device_bytes(self) -> int:
        return _lib.lib().rk_engine_device_bytes(self._h)

    def trace(self, program: int, max_ops: int = 512, max_ctas: int = 296):
        """Per-op stamps of one pass of a step program (rk_engine_trace): (stamps [n, 4] us, kinds [n],
        per-CTA [n, max_ctas, 2] us with -1 past the grid)."""
        st = (C.c_double * (4 * max_ops))()
        kd = (C.c_int * max_ops)()
        ct = (C.c_double * (2 * max_ops * max_ctas))()
        n = _lib.call("rk_engine_trace", self._h, program, st, kd, max_ops, ct, max_ctas)
        n = min(n, max_ops)
        return (np.frombuffer(st, dtype=np.float64)[:4 * n].reshape(n, 4).copy(),
                np.frombuffer(kd, dtype=np.int32)[:n].copy(),
                np.frombuffer(ct, dtype=np.float64)[:2 * n * max_ctas].reshape(n, max_ctas, 2).copy())

    @property
    def mode(self) -> str:
        """"persistent" (one cooperative kernel per step program) or "graph" (one kernel per op)."""
        return "persistent" if _lib.lib().rk_engine_mode(self._h) == 1 else "graph"
