"""ctypes bindings for the CPU oracle (``oracle/librefcpu.so``).

TEST INFRASTRUCTURE ONLY.  This module is the parity checker used by
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline / reference arm of
``bench.py``.  The product library never imports it, and nothing here is on
the measured GPU path.  The C sources (``refcpu.c``) say which reference
behaviour each function restates.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librefcpu.so")

QK = 32
Q4_0_BLOCK_BYTES = 18
Q8_0_BLOCK_BYTES = 34

_lib = None


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (gcc, OpenMP)."""
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(
        os.path.join(HERE, "refcpu.c")
    ):
        subprocess.run(["make", "-C", HERE, "-s"], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P = C.c_void_p
I64 = C.c_int64
I32 = C.c_int


def _declare(L):
    sig = {
        "ref_f16_to_f32": (C.c_float, [C.c_uint16]),
        "ref_f32_to_f16": (C.c_uint16, [C.c_float]),
        "ref_quantize_q8_0": (None, [P, P, I64]),
        "ref_quantize_q4_0": (None, [P, P, I64]),
        "ref_dequantize_q8_0": (None, [P, P, I64]),
        "ref_dequantize_q4_0": (None, [P, P, I64]),
        "ref_mul_mat_f16": (None, [P, P, P, I64, I64, I32]),
        "ref_mul_mat_q4_0": (None, [P, P, P, I64, I64, I32, I32]),
        "ref_mul_mat_q8_0": (None, [P, P, P, I64, I64, I32]),
        "ref_block_dots_q4_0": (None, [P, P, P, I64, I64]),
        "ref_mul_mat_q4_0_xq": (None, [P, P, P, I64, I64, I32]),
        "ref_block_dots_q4_0_xq": (None, [P, P, P, I64, I64]),
        "ref_block_dots_q8_0": (None, [P, P, P, I64, I64]),
        "ref_flash_attn_ext_decode": (
            None,
            [P, P, P, P, P, P, I32, I32, I32, I32, I64, I64, I64, I64, C.c_float, I32],
        ),
        "ref_kv_lengths_from_mask_f16": (None, [P, I64, I64, P]),
        "ref_a8w8_quantize_token": (None, [P, P, P, I64]),
        "ref_a8w8_transform_weight": (None, [P, P, P, I64, I64]),
        "ref_a8w8_matmul_i32": (None, [P, P, P, I64, I64]),
        "ref_a8w8_dequant": (None, [P, C.c_uint16, P, P, I64]),
        "ref_w4a16_probe": (None, [P, P, P, P, I64, I64, I64]),
        "ref_synth_normal": (C.c_float, [C.c_uint64, C.c_uint64]),
        "ref_synth_q4_0": (None, [C.c_uint64, C.c_float, I64, I64, I64, P, I32]),
        "ref_synth_rows_f16": (None, [C.c_uint64, C.c_uint64, I64, I64, I64, I64, P, I32]),
        "ref_rms_norm_mul": (None, [P, P, P, I64, C.c_float]),
        "ref_rope_norm": (None, [P, I32, I32, I32, C.c_float]),
        "ref_argmax": (I64, [P, I64]),
        "ref_llama_step": (I64, [P, C.c_int32, C.c_int32, P, P, I32, I32, I32, I32]),
        "ref_set_accum_mode": (None, [I32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(C.c_void_p)


# ----------------------------------------------------------------- blocks

def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """float32 [..., K] -> uint8 [..., K/32*34] ggml Q8_0 blocks."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = x.shape[-1]
    assert k % QK == 0
    out = np.empty(x.shape[:-1] + (k // QK * Q8_0_BLOCK_BYTES,), dtype=np.uint8)
    lib().ref_quantize_q8_0(_p(x), _p(out), x.size)
    return out


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = x.shape[-1]
    assert k % QK == 0
    out = np.empty(x.shape[:-1] + (k // QK * Q4_0_BLOCK_BYTES,), dtype=np.uint8)
    lib().ref_quantize_q4_0(_p(x), _p(out), x.size)
    return out


def dequantize_q8_0(b: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint8)
    nblk = b.size // Q8_0_BLOCK_BYTES
    out = np.empty(b.shape[:-1] + (b.shape[-1] // Q8_0_BLOCK_BYTES * QK,), dtype=np.float32)
    lib().ref_dequantize_q8_0(_p(b), _p(out), nblk * QK)
    return out


def dequantize_q4_0(b: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint8)
    nblk = b.size // Q4_0_BLOCK_BYTES
    out = np.empty(b.shape[:-1] + (b.shape[-1] // Q4_0_BLOCK_BYTES * QK,), dtype=np.float32)
    lib().ref_dequantize_q4_0(_p(b), _p(out), nblk * QK)
    return out


# ---------------------------------------------------------------- mul_mat

def mul_mat_f16(w: np.ndarray, x: np.ndarray, nthreads: int = 0) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.float16)
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, k = w.shape
    y = np.empty(n, dtype=np.float32)
    lib().ref_mul_mat_f16(_p(w), _p(x), _p(y), n, k, nthreads)
    return y


def mul_mat_q4_0(w_blocks: np.ndarray, x: np.ndarray, mode: int = 0, nthreads: int = 0) -> np.ndarray:
    w_blocks = np.ascontiguousarray(w_blocks, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = x.shape[-1]
    n = w_blocks.size // (k // QK * Q4_0_BLOCK_BYTES)
    y = np.empty(n, dtype=np.float32)
    lib().ref_mul_mat_q4_0(_p(w_blocks), _p(x), _p(y), n, k, mode, nthreads)
    return y


def mul_mat_q8_0(w_blocks: np.ndarray, x: np.ndarray, nthreads: int = 0) -> np.ndarray:
    w_blocks = np.ascontiguousarray(w_blocks, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = x.shape[-1]
    n = w_blocks.size // (k // QK * Q8_0_BLOCK_BYTES)
    y = np.empty(n, dtype=np.float32)
    lib().ref_mul_mat_q8_0(_p(w_blocks), _p(x), _p(y), n, k, nthreads)
    return y


def block_dots(fmt: str, w_blocks: np.ndarray, x: np.ndarray) -> np.ndarray:
    w_blocks = np.ascontiguousarray(w_blocks, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = x.shape[-1]
    bb = Q4_0_BLOCK_BYTES if fmt == "q4_0" else Q8_0_BLOCK_BYTES
    n = w_blocks.size // (k // QK * bb)
    dots = np.empty((n, k // QK), dtype=np.int32)
    fn = lib().ref_block_dots_q4_0 if fmt == "q4_0" else lib().ref_block_dots_q8_0
    fn(_p(w_blocks), _p(x), _p(dots), n, k)
    return dots


def mul_mat_q4_0_xq(w_blocks: np.ndarray, xq_blocks: np.ndarray, nthreads: int = 0) -> np.ndarray:
    """Q4_0 x Q8_0 MUL_MAT from given Q8_0 activation blocks (ggml-cpu after
    its src1 conversion): f32 [N]."""
    w_blocks = np.ascontiguousarray(w_blocks, dtype=np.uint8)
    xq_blocks = np.ascontiguousarray(xq_blocks, dtype=np.uint8)
    k = xq_blocks.size // Q8_0_BLOCK_BYTES * QK
    n = w_blocks.size // (k // QK * Q4_0_BLOCK_BYTES)
    y = np.empty(n, dtype=np.float32)
    lib().ref_mul_mat_q4_0_xq(_p(w_blocks), _p(xq_blocks), _p(y), n, k, nthreads)
    return y


def block_dots_q4_0_xq(w_blocks: np.ndarray, xq_blocks: np.ndarray) -> np.ndarray:
    """int32 [N, K/32] dots of Q4_0 rows with given Q8_0 activation blocks."""
    w_blocks = np.ascontiguousarray(w_blocks, dtype=np.uint8)
    xq_blocks = np.ascontiguousarray(xq_blocks, dtype=np.uint8)
    k = xq_blocks.size // Q8_0_BLOCK_BYTES * QK
    n = w_blocks.size // (k // QK * Q4_0_BLOCK_BYTES)
    dots = np.empty((n, k // QK), dtype=np.int32)
    lib().ref_block_dots_q4_0_xq(_p(w_blocks), _p(xq_blocks), _p(dots), n, k)
    return dots


def rms_norm_mul(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """ggml RMS_NORM (squares in f32, sum in double) followed by MUL."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    y = np.empty_like(x)
    lib().ref_rms_norm_mul(_p(x), _p(w), _p(y), x.size, C.c_float(eps))
    return y


def rope_norm(x: np.ndarray, n_heads: int, head_dim: int, pos: int, theta: float) -> np.ndarray:
    """ggml ROPE (NORM mode) of [n_heads * head_dim] f32 at one position."""
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    lib().ref_rope_norm(_p(y), n_heads, head_dim, pos, C.c_float(theta))
    return y


# -------------------------------------------------------------- attention

def flash_attn_decode(q, k, v, mask=None, kv_len=None, scale=None, mode=0):
    """q f32 [Hq, D]; k, v f16 [n_kv, Hkv, D] (token-major ggml cache view).

    Returns out f32 [Hq, D].  mode 0: fp64 truth; 1: ggml-cpu f16-V
    accumulation; 2: reference AttentionStepCustom (f16 output)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float16)
    v = np.ascontiguousarray(v, dtype=np.float16)
    hq, d = q.shape
    n_kv, hkv, d2 = k.shape
    assert d2 == d and v.shape == k.shape
    if scale is None:
        scale = 1.0 / np.sqrt(d)
    out = np.empty((hq, d), dtype=np.float32)
    mp = None
    if mask is not None:
        mask = np.ascontiguousarray(mask, dtype=np.float16)
        mp = _p(mask)
    lp = None
    if kv_len is not None:
        kl = np.ascontiguousarray(np.asarray([kv_len], dtype=np.int32))
        lp = _p(kl)
    lib().ref_flash_attn_ext_decode(
        _p(q), _p(k), _p(v), mp, lp, _p(out), d, hq, hkv, n_kv, hkv * d, d, hkv * d, d, float(scale), mode
    )
    return out


def kv_lengths_from_mask(mask_f16: np.ndarray) -> np.ndarray:
    m = np.ascontiguousarray(mask_f16, dtype=np.float16)
    if m.ndim == 1:
        m = m[None]
    out = np.empty(m.shape[0], dtype=np.int32)
    lib().ref_kv_lengths_from_mask_f16(_p(m), m.shape[1], m.shape[0], _p(out))
    return out


# ------------------------------------------------------- reference A8W8

def a8w8_quantize_token(x_f16: np.ndarray):
    x = np.ascontiguousarray(x_f16, dtype=np.float16)
    xq = np.empty(x.size, dtype=np.int8)
    s = np.empty(1, dtype=np.uint16)
    lib().ref_a8w8_quantize_token(_p(x), _p(xq), _p(s), x.size)
    return xq, s.view(np.float16)[0]


def a8w8_transform_weight(w_f16: np.ndarray):
    """w f16 [N][K] (ggml row n contiguous along K) -> (q_nz int8 [K*N], scales f16 [N])."""
    w = np.ascontiguousarray(w_f16, dtype=np.float16)
    n, k = w.shape
    q = np.empty(k * n, dtype=np.int8)
    s = np.empty(n, dtype=np.float16)
    lib().ref_a8w8_transform_weight(_p(w), _p(q), _p(s), k, n)
    return q, s


def a8w8_matmul_i32(xq, w_nz, k, n):
    acc = np.empty(n, dtype=np.int32)
    lib().ref_a8w8_matmul_i32(_p(np.ascontiguousarray(xq)), _p(np.ascontiguousarray(w_nz)), _p(acc), k, n)
    return acc


def a8w8_dequant(acc, x_scale_f16, w_scales_f16):
    acc = np.ascontiguousarray(acc, dtype=np.int32)
    ws = np.ascontiguousarray(w_scales_f16, dtype=np.float16)
    out = np.empty(acc.size, dtype=np.float16)
    xs = int(np.asarray(x_scale_f16, dtype=np.float16).view(np.uint16))
    lib().ref_a8w8_dequant(_p(acc), xs, _p(ws), _p(out), acc.size)
    return out


def a8w8_nz_index(kk, nn, k):
    """patch P:1690-1691 int8 NZ 16(K) x 32(N) element index."""
    return (((nn // 32) * (k // 16) + kk // 16) * 16 + kk % 16) * 32 + nn % 32


# ---------------------------------------------------- reference W4A16 probe

def w4a16_probe(x_f16, packed, scale_layout, k, n, tile=448):
    x = np.ascontiguousarray(x_f16, dtype=np.float16)
    pk = np.ascontiguousarray(packed, dtype=np.uint8)
    sl = np.ascontiguousarray(scale_layout, dtype=np.float16)
    y = np.empty(n, dtype=np.float16)
    lib().ref_w4a16_probe(_p(x), _p(pk), _p(sl), _p(y), k, n, tile)
    return y


# --------------------------------------------------------------- synthetic

def synth_q4_0(seed: int, sigma: float, row0: int, nrows: int, k: int, nthreads: int = 0) -> np.ndarray:
    out = np.empty((nrows, k // QK * Q4_0_BLOCK_BYTES), dtype=np.uint8)
    lib().ref_synth_q4_0(seed, sigma, row0, nrows, k, _p(out), nthreads)
    return out


def synth_rows_f16(seed: int, base: int, nrows: int, rl: int, rg: int | None = None, col0: int = 0,
                   nthreads: int = 0) -> np.ndarray:
    """f16 [nrows, rl] of the synthetic N(0,1) stream (the KV-cache fill)."""
    out = np.empty((nrows, rl), dtype=np.float16)
    lib().ref_synth_rows_f16(seed, base, nrows, rl, rl if rg is None else rg, col0, _p(out), nthreads)
    return out


def model_tensor_seed(seed: int, layer: int, which: int) -> int:
    """Seed of one weight tensor of the synthetic decode model (the native
    driver's tensor_seed): layer -1 for the embedding and the lm_head."""
    return (seed * 0x9E3779B97F4A7C15 + (layer + 2) * 0x100 + which) & 0xFFFFFFFFFFFFFFFF


def synth_llama_weights(cfg: dict, seed: int, sigma: float = 0.02, nthreads: int = 0) -> dict:
    """The synthetic decode model's weights (ggml Q4_0 rows, norms = 1) as
    b200_model_init_synthetic makes them on the device, regenerated on the
    host bit for bit (tensor parallel world 1)."""
    L, d, D = cfg["n_layer"], cfg["d_model"], cfg["head_dim"]
    qd, kvd, ff = cfg["n_head"] * D, cfg["n_head_kv"] * D, cfg["d_ff"]
    shapes = {"wq": (1, qd, d), "wk": (2, kvd, d), "wv": (3, kvd, d), "wo": (4, d, qd), "wgate": (5, ff, d),
              "wup": (6, ff, d), "wdown": (7, d, ff)}
    W = {"tok_embd": synth_q4_0(model_tensor_seed(seed, -1, 0), sigma, 0, cfg["vocab"], d, nthreads),
         "lm_head": synth_q4_0(model_tensor_seed(seed, -1, 8), sigma, 0, cfg["vocab"], d, nthreads)}
    for key, (which, rows, k) in shapes.items():
        W[key] = [synth_q4_0(model_tensor_seed(seed, l, which), sigma, 0, rows, k, nthreads) for l in range(L)]
    W["attn_norm"] = [np.ones(d, np.float32) for _ in range(L)]
    W["ffn_norm"] = [np.ones(d, np.float32) for _ in range(L)]
    W["out_norm"] = np.ones(d, np.float32)
    return W


def synth_llama_kv(cfg: dict, seed: int, n_pos: int, nthreads: int = 0):
    """KV caches [kv_size, n_head_kv * head_dim] f16 per layer, rows < n_pos
    filled as b200_model_fill_kv_synthetic does (world 1), the rest zero."""
    kvd = cfg["n_head_kv"] * cfg["head_dim"]
    kc, vc = [], []
    for l in range(cfg["n_layer"]):
        for w, dst in ((0, kc), (1, vc)):
            c = np.zeros((cfg["kv_size"], kvd), np.float16)
            if n_pos > 0:
                c[:n_pos] = synth_rows_f16(seed, (2 * l + w) << 40, n_pos, kvd, kvd, 0, nthreads)
            dst.append(c)
    return kc, vc


# ------------------------------------------------------------------ llama

class RefLlamaCfg(C.Structure):
    _fields_ = [
        ("n_layer", C.c_int), ("d_model", C.c_int), ("n_head", C.c_int), ("n_kv_head", C.c_int),
        ("head_dim", C.c_int), ("d_ff", C.c_int), ("vocab", C.c_int), ("kv_size", C.c_int),
        ("rope_theta", C.c_float), ("eps", C.c_float),
    ]


class RefLlama(C.Structure):
    _fields_ = [
        ("cfg", RefLlamaCfg),
        ("tok_embd", C.c_void_p),
        ("wq", C.POINTER(C.c_void_p)), ("wk", C.POINTER(C.c_void_p)), ("wv", C.POINTER(C.c_void_p)),
        ("wo", C.POINTER(C.c_void_p)),
        ("wgate", C.POINTER(C.c_void_p)), ("wup", C.POINTER(C.c_void_p)), ("wdown", C.POINTER(C.c_void_p)),
        ("attn_norm", C.POINTER(C.c_void_p)), ("ffn_norm", C.POINTER(C.c_void_p)),
        ("out_norm", C.c_void_p),
        ("lm_head", C.c_void_p),
        ("k_cache", C.POINTER(C.c_void_p)), ("v_cache", C.POINTER(C.c_void_p)),
    ]


class OracleLlama:
    """Holds numpy weights (ggml layouts) and runs ref_llama_step."""

    def __init__(self, cfg: dict, weights: dict, k_cache: list, v_cache: list):
        self.cfg = cfg
        self._keep = []
        L = cfg["n_layer"]

        def arr(lst):
            a = (C.c_void_p * L)(*[_p(t).value for t in lst])
            self._keep.append(a)
            return a

        for key in ("wq", "wk", "wv", "wo", "wgate", "wup", "wdown", "attn_norm", "ffn_norm"):
            for t in weights[key]:
                assert t.flags["C_CONTIGUOUS"]
        self.weights = weights
        self.k_cache = k_cache
        self.v_cache = v_cache
        m = RefLlama()
        m.cfg = RefLlamaCfg(
            cfg["n_layer"], cfg["d_model"], cfg["n_head"], cfg["n_head_kv"], cfg["head_dim"], cfg["d_ff"],
            cfg["vocab"], cfg["kv_size"], cfg["rope_theta"], cfg["rms_eps"],
        )
        m.tok_embd = _p(weights["tok_embd"]).value
        for key in ("wq", "wk", "wv", "wo", "wgate", "wup", "wdown", "attn_norm", "ffn_norm"):
            setattr(m, key, C.cast(arr(weights[key]), C.POINTER(C.c_void_p)))
        m.out_norm = _p(weights["out_norm"]).value
        m.lm_head = _p(weights["lm_head"]).value
        m.k_cache = C.cast(arr(k_cache), C.POINTER(C.c_void_p))
        m.v_cache = C.cast(arr(v_cache), C.POINTER(C.c_void_p))
        self.m = m
        self.x = np.zeros(cfg["d_model"], dtype=np.float32)
        self.logits = np.zeros(cfg["vocab"], dtype=np.float32)

    def step(self, token: int, pos: int, l0: int = 0, l1: int | None = None, do_head: bool = True,
             nthreads: int = 0) -> int:
        if l1 is None:
            l1 = self.cfg["n_layer"]
        return int(
            lib().ref_llama_step(C.byref(self.m), int(token), int(pos), _p(self.x), _p(self.logits), l0, l1,
                                 1 if do_head else 0, nthreads)
        )
