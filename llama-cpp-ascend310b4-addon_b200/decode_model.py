"""Python binding of the native decode driver (include/b200_model.h).

``DecodeModel`` owns a ``b200_model``: a Llama-architecture batch-1 decoder
with Q4_0 weights and an f16 KV cache, optionally tensor-parallel over the
GPUs of one node (one process per GPU, NCCL).  ``decode(token, pos)`` is the
end-to-end call a user makes (host token in, host token out); ``launch()``
replays the captured step on the device with the token fed back on the GPU.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

import b200_decode as B

W_TOK_EMBD, W_Q, W_K, W_V, W_O, W_GATE, W_UP, W_DOWN, W_LM_HEAD = range(9)
PROFILE_CLASSES = ["embed", "qkv", "attn", "o", "gate_up", "down", "lm_head", "allreduce"]


@dataclass
class LlamaConfig:
    n_layer: int
    d_model: int
    n_head: int
    n_head_kv: int
    head_dim: int
    d_ff: int
    vocab: int
    kv_size: int
    rope_theta: float = 500000.0
    rms_eps: float = 1e-5

    def as_dict(self):
        return dict(self.__dict__)


LLAMA3_70B = dict(n_layer=80, d_model=8192, n_head=64, n_head_kv=8, head_dim=128, d_ff=28672, vocab=128256,
                  rope_theta=500000.0, rms_eps=1e-5)


class _Cfg(C.Structure):
    _fields_ = [("n_layer", C.c_int), ("d_model", C.c_int), ("n_head", C.c_int), ("n_head_kv", C.c_int),
                ("head_dim", C.c_int), ("d_ff", C.c_int), ("vocab", C.c_int), ("kv_size", C.c_int),
                ("rope_theta", C.c_float), ("rms_eps", C.c_float)]


class _StepDump(C.Structure):
    _fields_ = [(name, C.c_void_p) for name in (
        "x", "x_mid", "q", "k_row", "v_row", "att", "h", "logits", "xq_qkv", "xq_o", "xq_gu", "xq_down", "xq_head",
        "dots_qkv", "dots_o", "dots_gu", "dots_down", "dots_head")]


DUMP_PARTS = [f for f, _ in _StepDump._fields_]

_declared = False


def _lib():
    global _declared
    L = B.lib()
    if not _declared:
        P = C.c_void_p
        sig = {
            "b200_nccl_unique_id": (C.c_int, [P]),
            "b200_model_create": (C.c_int, [C.POINTER(_Cfg), C.c_int, C.c_int, C.c_int, P, C.POINTER(P)]),
            "b200_model_destroy": (None, [P]),
            "b200_model_init_synthetic": (C.c_int, [P, C.c_uint64, C.c_float]),
            "b200_model_fill_kv_synthetic": (C.c_int, [P, C.c_uint64, C.c_int]),
            "b200_model_export_weight": (C.c_int, [P, C.c_int, C.c_int, P, C.POINTER(C.c_size_t)]),
            "b200_model_export_kv": (C.c_int, [P, C.c_int, C.c_int, C.c_int, P]),
            "b200_model_capture": (C.c_int, [P]),
            "b200_model_set_state": (C.c_int, [P, C.c_int, C.c_int, C.c_int]),
            "b200_model_launch": (C.c_int, [P]),
            "b200_model_decode": (C.c_int, [P, C.c_int, C.c_int, C.POINTER(C.c_int), P]),
            "b200_model_logits": (C.c_int, [P, P, C.POINTER(C.c_int64), C.POINTER(C.c_int64)]),
            "b200_model_stream": (P, [P]),
            "b200_model_step_bytes": (C.c_int, [P, C.c_int, C.POINTER(C.c_uint64)]),
            "b200_model_profile": (C.c_int, [P, C.c_int, P]),
            "b200_model_time_gate_up": (C.c_int, [P, C.c_int, C.POINTER(C.c_float)]),
            "b200_model_debug_step": (C.c_int, [P, C.c_int, C.c_int, P, P, P]),
            "b200_model_debug_step_ex": (C.c_int, [P, C.c_int, C.c_int, C.POINTER(_StepDump)]),
            "b200_model_timeline": (C.c_int, [P, P]),
            "b200_model_timeline_phases": (C.c_int, [P, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _declared = True
    return L


def nccl_unique_id() -> bytes:
    buf = (C.c_ubyte * 128)()
    B._check(_lib().b200_nccl_unique_id(C.cast(buf, C.c_void_p)), "nccl_unique_id")
    return bytes(buf)


class DecodeModel:
    def __init__(self, cfg: LlamaConfig, device: int = 0, tp_rank: int = 0, tp_world: int = 1,
                 nccl_id: bytes | None = None):
        self.cfg = cfg
        self.tp_rank, self.tp_world = tp_rank, tp_world
        c = _Cfg(cfg.n_layer, cfg.d_model, cfg.n_head, cfg.n_head_kv, cfg.head_dim, cfg.d_ff, cfg.vocab,
                 cfg.kv_size, cfg.rope_theta, cfg.rms_eps)
        h = C.c_void_p()
        idbuf = None
        if nccl_id is not None:
            idbuf = (C.c_ubyte * 128).from_buffer_copy(nccl_id)
        rc = _lib().b200_model_create(C.byref(c), device, tp_rank, tp_world,
                                      C.cast(idbuf, C.c_void_p) if idbuf is not None else None, C.byref(h))
        B._check(rc, "b200_model_create")
        self.h = h
        self._next = C.c_int(0)

    def close(self):
        if self.h:
            _lib().b200_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- setup
    def init_synthetic(self, seed: int = 1234, sigma: float = 0.02):
        B._check(_lib().b200_model_init_synthetic(self.h, seed, sigma), "init_synthetic")

    def fill_kv_synthetic(self, seed: int, n_pos: int):
        B._check(_lib().b200_model_fill_kv_synthetic(self.h, seed, n_pos), "fill_kv_synthetic")

    def export_weight(self, which: int, layer: int = -1) -> np.ndarray:
        n = C.c_size_t(0)
        B._check(_lib().b200_model_export_weight(self.h, layer, which, None, C.byref(n)), "export_weight")
        out = np.empty(n.value, dtype=np.uint8)
        B._check(_lib().b200_model_export_weight(self.h, layer, which, out.ctypes.data_as(C.c_void_p),
                                                 C.byref(n)), "export_weight")
        return out

    def export_kv(self, layer: int, which: int, n_pos: int) -> np.ndarray:
        kvd = self.cfg.n_head_kv // self.tp_world * self.cfg.head_dim
        out = np.empty((max(n_pos, 0), kvd), dtype=np.float16)
        B._check(_lib().b200_model_export_kv(self.h, layer, which, n_pos, out.ctypes.data_as(C.c_void_p)),
                 "export_kv")
        return out

    def capture(self):
        B._check(_lib().b200_model_capture(self.h), "capture")

    # ---- stepping
    def set_state(self, token: int, pos: int, advance: bool = True):
        B._check(_lib().b200_model_set_state(self.h, token, pos, 1 if advance else 0), "set_state")

    def launch(self):
        B._check(_lib().b200_model_launch(self.h), "launch")

    def decode(self, token: int, pos: int, want_logits: bool = False):
        """End to end: token/pos from the host, next token back to the host."""
        logits = None
        lp = None
        if want_logits:
            logits = np.empty(self.cfg.vocab // self.tp_world, dtype=np.float32)
            lp = logits.ctypes.data_as(C.c_void_p)
        B._check(_lib().b200_model_decode(self.h, token, pos, C.byref(self._next), lp), "decode")
        return (self._next.value, logits) if want_logits else self._next.value

    def logits(self):
        off, cnt = C.c_int64(0), C.c_int64(0)
        B._check(_lib().b200_model_logits(self.h, None, C.byref(off), C.byref(cnt)), "logits")
        out = np.empty(cnt.value, dtype=np.float32)
        B._check(_lib().b200_model_logits(self.h, out.ctypes.data_as(C.c_void_p), None, None), "logits")
        return off.value, out

    def stream_handle(self) -> int:
        return int(_lib().b200_model_stream(self.h) or 0)

    def step_bytes(self, ctx: int) -> int:
        v = C.c_uint64(0)
        B._check(_lib().b200_model_step_bytes(self.h, ctx, C.byref(v)), "step_bytes")
        return int(v.value)

    def debug_step(self, token: int, pos: int):
        """Layer dump of one eager step: x after embedding and after every
        layer [(L+1), d], roped q [L, Hq*D] and attention output [L, Hq*D]."""
        c = self.cfg
        hqd = c.n_head // self.tp_world * c.head_dim
        x = np.empty((c.n_layer + 1, c.d_model), np.float32)
        q = np.empty((c.n_layer, hqd), np.float32)
        a = np.empty((c.n_layer, hqd), np.float32)
        B._check(_lib().b200_model_debug_step(self.h, token, pos, x.ctypes.data_as(C.c_void_p),
                                              q.ctypes.data_as(C.c_void_p), a.ctypes.data_as(C.c_void_p)),
                 "debug_step")
        return x, q, a

    def dump_step(self, token: int, pos: int, parts=None) -> dict:
        """Full layer dump of one eager step (b200_model_debug_step_ex):
        every stage output and every Q8_0 activation (ggml block_q8_0 bytes)
        and per-block int32 dot array the step's GEMVs used.  `parts` names
        the entries to fetch (default: all of DUMP_PARTS)."""
        c = self.cfg
        w = self.tp_world
        L, d, D = c.n_layer, c.d_model, c.head_dim
        hq, hkv, ff, voc = c.n_head // w, c.n_head_kv // w, c.d_ff // w, c.vocab // w
        qd, kvd = hq * D, hkv * D
        qkv_rows = qd + 2 * kvd
        shapes = {
            "x": ((L + 1, d), np.float32), "x_mid": ((L, d), np.float32), "q": ((L, qd), np.float32),
            "k_row": ((L, kvd), np.float16), "v_row": ((L, kvd), np.float16), "att": ((L, qd), np.float32),
            "h": ((L, ff), np.float32), "logits": ((voc,), np.float32),
            "xq_qkv": ((L, d // 32 * 34), np.uint8), "xq_o": ((L, qd // 32 * 34), np.uint8),
            "xq_gu": ((L, d // 32 * 34), np.uint8), "xq_down": ((L, ff // 32 * 34), np.uint8),
            "xq_head": ((d // 32 * 34,), np.uint8),
            "dots_qkv": ((L, qkv_rows, d // 32), np.int32), "dots_o": ((L, d, qd // 32), np.int32),
            "dots_gu": ((L, 2 * ff, d // 32), np.int32), "dots_down": ((L, d, ff // 32), np.int32),
            "dots_head": ((voc, d // 32), np.int32),
        }
        want = DUMP_PARTS if parts is None else list(parts)
        out, sd = {}, _StepDump()
        for name in want:
            shape, dt = shapes[name]
            out[name] = np.empty(shape, dtype=dt)
            setattr(sd, name, out[name].ctypes.data_as(C.c_void_p).value)
        B._check(_lib().b200_model_debug_step_ex(self.h, token, pos, C.byref(sd)), "debug_step_ex")
        return out

    def timeline(self) -> dict:
        """In-step time per kernel class of one captured step
        (b200_model_timeline): {"step_us", "advance_us": {class: us},
        "span_us": {class: mean us per kernel}, "phases_us": {class: {mark:
        us after the class's wait}}} (b200_model_timeline_phases)."""
        out = (C.c_float * 17)()
        B._check(_lib().b200_model_timeline(self.h, C.cast(out, C.c_void_p)), "timeline")
        ph = (C.c_float * 64)()
        B._check(_lib().b200_model_timeline_phases(self.h, C.cast(ph, C.c_void_p)), "timeline_phases")
        marks = ("resident_before_wait", "input_ready", "first_chunk", "loop_done", "exit",
                 "input_ready_first_cta", "first_chunk_first_cta", "loop_done_first_cta")
        return {"step_us": float(out[16]),
                "advance_us": {k: float(out[i]) for i, k in enumerate(PROFILE_CLASSES) if i > 0},
                "span_us": {k: float(out[8 + i]) for i, k in enumerate(PROFILE_CLASSES) if i > 0},
                "phases_us": {k: {mk: round(float(ph[8 * i + j]), 2) for j, mk in enumerate(marks)}
                              for i, k in enumerate(PROFILE_CLASSES) if i > 0}}

    def time_gate_up(self, iters: int = 5) -> float:
        """us per gate/up GEMV launch, from a graph of the step's n_layer
        gate/up launches (overwrites the step's SwiGLU scratch)."""
        us = C.c_float(0.0)
        B._check(_lib().b200_model_time_gate_up(self.h, iters, C.byref(us)), "time_gate_up")
        return float(us.value)

    def profile(self, iters: int = 3) -> dict:
        us = (C.c_float * 8)()
        B._check(_lib().b200_model_profile(self.h, iters, C.cast(us, C.c_void_p)), "profile")
        return {k: float(us[i]) for i, k in enumerate(PROFILE_CLASSES)}


def oracle_weights(model: DecodeModel):
    """The model's weights in ggml layout on the host (test infrastructure:
    feeds the CPU oracle).  Only for tp_world == 1."""
    cfg = model.cfg
    L = cfg.n_layer
    w = {"tok_embd": model.export_weight(W_TOK_EMBD), "lm_head": model.export_weight(W_LM_HEAD)}
    for key, which in (("wq", W_Q), ("wk", W_K), ("wv", W_V), ("wo", W_O), ("wgate", W_GATE), ("wup", W_UP),
                       ("wdown", W_DOWN)):
        w[key] = [model.export_weight(which, l) for l in range(L)]
    w["attn_norm"] = [np.ones(cfg.d_model, np.float32) for _ in range(L)]
    w["ffn_norm"] = [np.ones(cfg.d_model, np.float32) for _ in range(L)]
    w["out_norm"] = np.ones(cfg.d_model, np.float32)
    return w
