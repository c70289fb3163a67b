"""Python host-side binding of libb200_decode.so (ctypes over the C ABI).

The functions mirror the ggml ops this backend serves, with ggml's argument
meaning: ``mul_mat(w, x)`` is ggml_mul_mat(src0=W[K, N], src1=x[K, 1]) -> f32
[N], and ``flash_attn_ext(q, k, v, mask, scale, ...)`` is
ggml_flash_attn_ext for one query token with the reference add-on's optional
``kv_lengths`` source (ggml_flash_attn_ext_add_kv_lengths, patch:2009-2023).
Contract violations raise ``B200Error`` (the reference aborts through
GGML_ASSERT); unsupported variants raise ``B200Unsupported`` so a caller can
route them elsewhere, as ggml's scheduler does when supports_op is false.

Tensors are torch CUDA tensors; torch is used only to hold device memory and
to name the current stream.  There is no CPU fallback: when the shared
library is missing this module raises on import of the library.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libb200_decode.so")

TYPE_F32 = 0
TYPE_F16 = 1
TYPE_Q4_0 = 2
TYPE_Q8_0 = 8
TYPE_A8W8 = 100  # this library's int8 layout for the reference's A8W8 scheme
Q4_MODE_GGML = 0
Q4_MODE_W4A16 = 1

BLOCK_BYTES = {TYPE_Q4_0: 18, TYPE_Q8_0: 34}

OK = 0
EINVAL = -1
ECUDA = -2
EUNSUPPORTED = -3
ESCRATCH = -7
FA_STATIC_SCRATCH_BYTES = 4 << 20

_lib = None


class B200Error(RuntimeError):
    def __init__(self, code: int, what: str):
        self.code = code
        super().__init__(f"{what}: {lib().b200_strerror(code).decode()} ({code})")


class B200Unsupported(B200Error):
    pass


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing; build it with `python {os.path.join(HERE, 'build.py')}` "
                "(there is no fallback path)"
            )
        # torch first: its bundled NCCL must own the libnccl.so.2 soname.  The
        # library links NCCL too; loaded first, it would bring the system's
        # older NCCL, which a later `import torch` then fails to bind to.
        try:
            import torch  # noqa: F401
        except ImportError:
            pass
        _lib = C.CDLL(LIB_PATH, mode=C.RTLD_GLOBAL)
        _declare(_lib)
    return _lib


P = C.c_void_p
I64 = C.c_int64


def _declare(L):
    sig = {
        "b200_version": (C.c_char_p, []),
        "b200_strerror": (C.c_char_p, [C.c_int]),
        "b200_device_status": (C.c_int, [C.POINTER(C.c_uint), C.c_int]),
        "b200_set_wait_timeout": (C.c_int, [C.c_uint64]),
        "b200_tp_allreduce_f32": (C.c_int, [P, C.POINTER(P), C.c_int, C.c_int, I64, P, C.POINTER(P), C.c_uint64, P]),
        "b200_packed_row_stride": (I64, [C.c_int, I64, I64]),
        "b200_packed_size": (C.c_size_t, [C.c_int, I64, I64]),
        "b200_repack": (C.c_int, [C.c_int, P, P, I64, I64, P]),
        "b200_repack_interleave2": (C.c_int, [C.c_int, P, P, P, I64, I64, P]),
        "b200_gemv_f16": (C.c_int, [P, P, P, I64, I64, P]),
        "b200_mul_mat_f16": (C.c_int, [P, P, P, I64, I64, C.c_int, I64, I64, P]),
        "b200_mul_mat_f16_tc_workspace_size": (C.c_size_t, [I64, I64]),
        "b200_mul_mat_f16_tc": (C.c_int, [P, P, P, I64, I64, I64, I64, I64, P, C.c_size_t, P]),
        "b200_gemv_q4_0": (C.c_int, [P, P, P, I64, I64, C.c_int, P]),
        "b200_gemv_q8_0_q8_0": (C.c_int, [P, P, P, I64, I64, P]),
        "b200_a8w8_transform": (C.c_int, [P, P, I64, I64, P]),
        "b200_gemv_a8w8": (C.c_int, [P, P, P, I64, I64, P]),
        "b200_a8w8_selects_weight": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(I64), C.c_char_p, C.c_int]),
        "b200_quantize_q8_0": (C.c_int, [P, P, I64, P]),
        "b200_gemv_block_dots": (C.c_int, [C.c_int, P, P, P, P, I64, I64, P]),
        "b200_fa_workspace_size": (C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int]),
        "b200_fa_decode": (
            C.c_int,
            [P, P, P, P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, I64, I64, I64, I64, C.c_float, P, C.c_size_t, P],
        ),
        "b200_fa_decode_static_scratch": (
            C.c_int,
            [P, P, P, P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, I64, I64, I64, I64, C.c_float, P],
        ),
        "b200_kv_lengths_from_mask_f16": (C.c_int, [P, I64, I64, P]),
        "b200_rms_norm_f32": (C.c_int, [P, P, P, I64, I64, C.c_float, P]),
        "b200_rope_norm_f32": (C.c_int, [P, P, P, I64, C.c_int, C.c_int, C.c_float, P]),
        "b200_set_rows_f16": (C.c_int, [P, P, P, I64, I64, I64, I64, P]),
        "b200_get_rows_q4_0": (C.c_int, [P, P, P, I64, I64, I64, P]),
        "b200_get_rows_q4_0_packed": (C.c_int, [P, P, P, I64, I64, I64, P]),
        "b200_upload_begin": (C.c_int, [C.c_int, I64, I64, P, C.POINTER(P)]),
        "b200_upload_write": (C.c_int, [P, C.c_size_t, P, C.c_size_t, C.POINTER(C.c_int)]),
        "b200_upload_end": (C.c_int, [P]),
        "b200_swiglu_f32": (C.c_int, [P, P, P, I64, P]),
        "b200_add_f32": (C.c_int, [P, P, P, I64, P]),
        "b200_argmax_f32": (C.c_int, [P, I64, P, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _check(rc: int, what: str):
    if rc == EUNSUPPORTED:
        raise B200Unsupported(rc, what)
    if rc != OK:
        raise B200Error(rc, what)


def _torch():
    import torch

    return torch


def _stream(device=None):
    torch = _torch()
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def device_status(reset: bool = True) -> int:
    v = C.c_uint(0)
    _check(lib().b200_device_status(C.byref(v), 1 if reset else 0), "b200_device_status")
    return int(v.value)


DEVSTATUS_TIMEOUT = 1
DEVSTATUS_BOUNDS = 2


def set_wait_timeout(ns: int = 0):
    """Limit of every bounded device-side wait on the current device (0: the
    default 2 s)."""
    _check(lib().b200_set_wait_timeout(int(ns)), "b200_set_wait_timeout")


def tp_allreduce_f32(x, parts, rank: int, flags, peer_flags, seq: int, stream=None):
    """One-shot peer-memory all-reduce (sum in rank order) of n floats.

    x: f32 [n] device tensor (result); parts: world device pointers (ints)
    or tensors holding every rank's partial; flags: this rank's u64 flag
    array [world]; peer_flags: world device addresses of
    &flags_of_rank_r[rank]; seq: collective number (> 0, increasing)."""
    torch = _torch()
    world = len(parts)
    if len(peer_flags) != world:
        raise B200Error(EINVAL, "tp_allreduce_f32: parts and peer_flags differ in length")
    if x.dtype != torch.float32 or not x.is_contiguous() or not x.is_cuda:
        raise B200Error(EINVAL, "tp_allreduce_f32: x must be a contiguous f32 CUDA tensor")

    def addr(p):
        return int(p.data_ptr()) if hasattr(p, "data_ptr") else int(p)

    pa = (P * world)(*[addr(p) for p in parts])
    fa = (P * world)(*[addr(p) for p in peer_flags])
    st = C.c_void_p(stream) if stream is not None else _stream(x.device)
    _check(lib().b200_tp_allreduce_f32(_ptr(x), pa, world, rank, x.numel(), C.c_void_p(addr(flags)), fa, int(seq),
                                       st), "tp_allreduce_f32")
    return x


# ----------------------------------------------------------- packed weights

def packed_size(wtype: int, n: int, k: int) -> int:
    return int(lib().b200_packed_size(wtype, n, k))


def row_stride(wtype: int, n: int, k: int) -> int:
    return int(lib().b200_packed_row_stride(wtype, n, k))


class PackedWeight:
    """A weight in the tile-interleaved layout on the device."""

    def __init__(self, wtype: int, n: int, k: int, data):
        self.wtype, self.n, self.k, self.data = wtype, n, k, data


def repack(wtype: int, src, n: int, k: int) -> PackedWeight:
    """src: device tensor holding ggml rows (F16 [n, k] or Q4_0/Q8_0 block bytes)."""
    torch = _torch()
    size = packed_size(wtype, n, k)
    if size == 0:
        raise B200Unsupported(EUNSUPPORTED, f"repack type={wtype} n={n} k={k}")
    dst = torch.empty(size, dtype=torch.uint8, device=src.device)
    _check(lib().b200_repack(wtype, _ptr(src), _ptr(dst), n, k, _stream(src.device)), "b200_repack")
    return PackedWeight(wtype, n, k, dst)


def a8w8_selects_weight(name: str, wtype: int, ne, disable_layers: str | None = None,
                        tied_output: bool = False) -> bool:
    """The reference's A8W8 weight policy (ggml_cann_310b_is_a8w8_weight,
    patch:1520-1533, with GGML_CANN_A8W8_DISABLE_LAYERS parsed as in
    ggml_cann_310b_a8w8_layer_disabled, patch:1481-1514): True for an F16
    FFN gate/up/down weight of a layer not in `disable_layers`, or the tied
    1536 x 151936 token_embd.weight when `tied_output`."""
    arr = (C.c_int64 * 4)(*[int(v) for v in (list(ne) + [1, 1, 1, 1])[:4]])
    dl = disable_layers.encode() if disable_layers is not None else None
    rc = lib().b200_a8w8_selects_weight(name.encode(), int(wtype), arr, dl, 1 if tied_output else 0)
    if rc < 0:
        _check(rc, "b200_a8w8_selects_weight")
    return rc == 1


def a8w8_transform(w_f16, n: int, k: int) -> PackedWeight:
    """The reference's F16 -> A8W8 weight transform (per-row int8 + f16 scale)
    of a ggml F16 weight [n, k] on the device."""
    torch = _torch()
    dst = torch.empty(packed_size(TYPE_A8W8, n, k), dtype=torch.uint8, device=w_f16.device)
    _check(lib().b200_a8w8_transform(_ptr(w_f16.contiguous()), _ptr(dst), n, k, _stream(w_f16.device)),
           "b200_a8w8_transform")
    return PackedWeight(TYPE_A8W8, n, k, dst)


def repack_interleave2(wtype: int, src_even, src_odd, n_each: int, k: int) -> PackedWeight:
    torch = _torch()
    size = packed_size(wtype, 2 * n_each, k)
    dst = torch.empty(size, dtype=torch.uint8, device=src_even.device)
    _check(
        lib().b200_repack_interleave2(wtype, _ptr(src_even), _ptr(src_odd), _ptr(dst), n_each, k,
                                      _stream(src_even.device)),
        "b200_repack_interleave2",
    )
    return PackedWeight(wtype, 2 * n_each, k, dst)


# ------------------------------------------------------------------ mul_mat

def mul_mat(w: PackedWeight, x, y=None, q4_mode: int = Q4_MODE_GGML):
    """ggml_mul_mat(W, x): x f32 [K] -> y f32 [N] (M = 1, every weight type),
    or x f32 [M, K] -> y f32 [M, N] for M <= 8 columns (F16 weights: the
    reference's small-M NZ branch)."""
    torch = _torch()
    if x.dim() == 2 and x.shape[0] > 1:
        if w.wtype != TYPE_F16:
            raise B200Unsupported(EUNSUPPORTED, f"mul_mat with {x.shape[0]} columns for weight type {w.wtype}")
        assert x.dtype == torch.float32 and x.stride(1) == 1 and x.shape[1] == w.k
        m = x.shape[0]
        if y is None:
            y = torch.empty(m, w.n, dtype=torch.float32, device=x.device)
        if m > 8:  # prefill: the tensor-core GEMM (the packed F16 layout is the ggml row layout)
            return mul_mat_f16_tc(w.data, x, w.n, w.k, y)
        rc = lib().b200_mul_mat_f16(_ptr(w.data), _ptr(x), _ptr(y), w.n, w.k, m, x.stride(0), y.stride(0),
                                    _stream(x.device))
        _check(rc, "mul_mat")
        return y
    assert x.dtype == torch.float32 and x.is_contiguous() and x.numel() == w.k
    if y is None:
        y = torch.empty(w.n, dtype=torch.float32, device=x.device)
    s = _stream(x.device)
    if w.wtype == TYPE_F16:
        rc = lib().b200_gemv_f16(_ptr(w.data), _ptr(x), _ptr(y), w.n, w.k, s)
    elif w.wtype == TYPE_Q4_0:
        rc = lib().b200_gemv_q4_0(_ptr(w.data), _ptr(x), _ptr(y), w.n, w.k, q4_mode, s)
    elif w.wtype == TYPE_Q8_0:
        rc = lib().b200_gemv_q8_0_q8_0(_ptr(w.data), _ptr(x), _ptr(y), w.n, w.k, s)
    elif w.wtype == TYPE_A8W8:
        rc = lib().b200_gemv_a8w8(_ptr(w.data), _ptr(x), _ptr(y), w.n, w.k, s)
    else:
        raise B200Unsupported(EUNSUPPORTED, f"mul_mat weight type {w.wtype}")
    _check(rc, "mul_mat")
    return y


_tc_ws: dict = {}


def mul_mat_f16_tc(w_f16, x, n: int, k: int, y=None):
    """Prefill MUL_MAT of an F16 weight ([n, k] ggml rows on the device) with
    x f32 [m, k] (row stride >= k) on the tcgen05 tensor cores -> y f32 [m, n].
    The f16 copy of x goes to a workspace cached per device and size."""
    torch = _torch()
    m = x.shape[0]
    if x.dtype != torch.float32 or x.stride(1) != 1 or x.shape[1] != k:
        raise B200Error(EINVAL, "mul_mat_f16_tc: x must be f32 [m, k] with a contiguous row")
    if y is None:
        y = torch.empty(m, n, dtype=torch.float32, device=x.device)
    size = int(lib().b200_mul_mat_f16_tc_workspace_size(m, k))
    key = (str(x.device), size)
    ws = _tc_ws.get(key)
    if ws is None:
        ws = torch.empty(size, dtype=torch.uint8, device=x.device)
        _tc_ws[key] = ws
    rc = lib().b200_mul_mat_f16_tc(_ptr(w_f16), _ptr(x), _ptr(y), n, k, m, x.stride(0), y.stride(0), _ptr(ws), size,
                                   _stream(x.device))
    _check(rc, "mul_mat_f16_tc")
    return y


def quantize_q8_0(x):
    torch = _torch()
    k = x.numel()
    out = torch.empty(k // 32 * 34, dtype=torch.uint8, device=x.device)
    _check(lib().b200_quantize_q8_0(_ptr(x), _ptr(out), k, _stream(x.device)), "quantize_q8_0")
    return out


def block_dots(w: PackedWeight, x, with_activation: bool = False):
    """Runs the GEMV kernel in its export mode: int32 dots [N, K/32] and,
    optionally, the Q8_0 blocks its prologue produced from x."""
    torch = _torch()
    dots = torch.empty((w.n, w.k // 32), dtype=torch.int32, device=x.device)
    xq = torch.empty(w.k // 32 * 34, dtype=torch.uint8, device=x.device) if with_activation else None
    _check(lib().b200_gemv_block_dots(w.wtype, _ptr(w.data), _ptr(x), _ptr(dots), _ptr(xq), w.n, w.k,
                                      _stream(x.device)), "block_dots")
    return (dots, xq) if with_activation else dots


# ------------------------------------------------------------ attention

_ws_cache: dict = {}


def fa_workspace(head_dim: int, n_head: int, n_head_kv: int, n_kv: int, device):
    torch = _torch()
    size = int(lib().b200_fa_workspace_size(head_dim, n_head, n_head_kv, n_kv))
    if size == 0:
        raise B200Error(EINVAL, "fa_workspace_size")
    key = (str(device), size)
    ws = _ws_cache.get(key)
    if ws is None:
        ws = torch.zeros(size, dtype=torch.uint8, device=device)
        _ws_cache[key] = ws
    return ws


def _check_fa_tensors(what, q, k, v, mask, kv_lengths, out):
    """The op contract of FLASH_ATTN_EXT at one query token (the reference
    asserts the same types, patch:1378-1382 and patch:2017-2020): q f32
    [Hq, D]; k, v f16 [n_kv, Hkv, D] with a contiguous head dim; mask f16
    with at least n_kv entries; kv_lengths int32 with at least one; out f32
    [Hq, D] contiguous; all on q's device.  Returns (hq, d, n_kv, hkv)."""
    torch = _torch()

    def bad(msg):
        raise B200Error(EINVAL, f"{what}: {msg}")

    if q.dim() != 2 or k.dim() != 3 or v.dim() != 3:
        bad("q must be [Hq, D] and k, v [n_kv, Hkv, D]")
    hq, d = q.shape
    n_kv, hkv, d2 = k.shape
    if d2 != d or tuple(v.shape) != tuple(k.shape):
        bad("shapes")
    if q.dtype != torch.float32 or k.dtype != torch.float16 or v.dtype != torch.float16:
        bad("q must be f32 and k, v f16")
    dev = q.device
    if not q.is_cuda or k.device != dev or v.device != dev:
        bad("q, k, v must be on one CUDA device")
    if k.stride(2) != 1 or v.stride(2) != 1:
        bad("needs contiguous head dim")
    if mask is not None and (mask.dtype != torch.float16 or mask.device != dev or not mask.is_contiguous()
                             or mask.numel() < n_kv):
        bad("mask must be a contiguous f16 tensor of at least n_kv entries on q's device")
    if kv_lengths is not None and (kv_lengths.dtype != torch.int32 or kv_lengths.device != dev
                                   or kv_lengths.numel() < 1):
        bad("kv_lengths must be an int32 tensor on q's device")
    if out is not None and (out.dtype != torch.float32 or out.device != dev or not out.is_contiguous()
                            or tuple(out.shape) != (hq, d)):
        bad("out must be a contiguous f32 [Hq, D] tensor on q's device")
    return hq, d, n_kv, hkv


def flash_attn_ext(q, k, v, mask=None, scale: float = 1.0, max_bias: float = 0.0, logit_softcap: float = 0.0,
                   kv_lengths=None, out=None, workspace=None):
    """ggml_flash_attn_ext for one query token.

    q f32 [Hq, D]; k, v f16 tensors viewed as [n_kv, Hkv, D] (any strides with
    a contiguous last dim); mask f16 [n_kv] or None; kv_lengths int32 [>=1]
    device tensor or None.  Returns f32 [Hq, D]."""
    torch = _torch()
    if max_bias != 0.0 or logit_softcap != 0.0:
        raise B200Unsupported(EUNSUPPORTED, "flash_attn_ext with ALiBi or softcap")
    hq, d, n_kv, hkv = _check_fa_tensors("flash_attn_ext", q, k, v, mask, kv_lengths, out)
    q = q.contiguous()
    if out is None:
        out = torch.empty((hq, d), dtype=torch.float32, device=q.device)
    if workspace is None:
        workspace = fa_workspace(d, hq, hkv, n_kv, q.device)
    es = k.element_size()
    rc = lib().b200_fa_decode(
        _ptr(q), _ptr(k), _ptr(v), _ptr(mask), _ptr(kv_lengths), _ptr(out), d, hq, hkv, n_kv,
        k.stride(0) * es, k.stride(1) * es, v.stride(0) * es, v.stride(1) * es, float(scale),
        _ptr(workspace), workspace.numel(), _stream(q.device),
    )
    _check(rc, "flash_attn_ext")
    return out


def flash_attn_ext_static_scratch(q, k, v, mask=None, scale: float = 1.0, kv_lengths=None, out=None):
    """flash_attn_ext that allocates nothing on the device.

    For hosts that cannot hand over or allocate a workspace: the partials go
    to the library's fixed per-device static array (FA_STATIC_SCRATCH_BYTES).
    Calls larger than that raise B200Error(ESCRATCH); calls that overlap on
    one GPU share the array and race.  Only ``out`` may be allocated here, and
    only when the caller passes none."""
    torch = _torch()
    hq, d, n_kv, hkv = _check_fa_tensors("flash_attn_ext_static_scratch", q, k, v, mask, kv_lengths, out)
    if not q.is_contiguous():
        raise B200Error(EINVAL, "flash_attn_ext_static_scratch needs a contiguous q")
    if out is None:
        out = torch.empty((hq, d), dtype=torch.float32, device=q.device)
    es = k.element_size()
    rc = lib().b200_fa_decode_static_scratch(
        _ptr(q), _ptr(k), _ptr(v), _ptr(mask), _ptr(kv_lengths), _ptr(out), d, hq, hkv, n_kv,
        k.stride(0) * es, k.stride(1) * es, v.stride(0) * es, v.stride(1) * es, float(scale), _stream(q.device),
    )
    _check(rc, "flash_attn_ext_static_scratch")
    return out


# ------------------------------------------------------------ neighbour ops
# ggml's RMS_NORM (+ MUL), ROPE (NORM mode), SET_ROWS, GET_ROWS, SWIGLU, ADD
# and ARGMAX for a backend that runs the decode graph op by op.


def rms_norm(x, eps: float, w=None, out=None):
    """x f32 [rows, n] (or [n]); y = x / sqrt(mean(x^2) + eps) * w."""
    torch = _torch()
    x = x.contiguous()
    n = x.shape[-1]
    rows = x.numel() // n
    out = torch.empty_like(x) if out is None else out
    _check(lib().b200_rms_norm_f32(_ptr(x), _ptr(w), _ptr(out), n, rows, float(eps), _stream(x.device)), "rms_norm")
    return out


def rope_norm(x, pos, freq_base: float, out=None):
    """x f32 [n_tokens, n_heads, head_dim]; pos int32 [n_tokens] on the device."""
    torch = _torch()
    x = x.contiguous()
    n_tokens, n_heads, head_dim = x.shape
    out = torch.empty_like(x) if out is None else out
    _check(lib().b200_rope_norm_f32(_ptr(x), _ptr(out), _ptr(pos), n_tokens, n_heads, head_dim, float(freq_base),
                                    _stream(x.device)), "rope_norm")
    return out


def set_rows_f16(src, idx, dst):
    """dst[idx[r], :n] = f16(src[r]); dst f16 [rows, >= n] (row-strided view), idx int64."""
    nrows, n = src.shape
    _check(lib().b200_set_rows_f16(_ptr(src.contiguous()), _ptr(idx), _ptr(dst), n, nrows, dst.stride(0) * 2,
                                   dst.shape[0], _stream(src.device)), "set_rows_f16")
    return dst


def get_rows_q4_0(table, idx, vocab: int, n: int, out=None):
    """table: Q4_0 blocks [vocab, n/32 * 18] (ggml layout); idx int32 [nidx] -> f32 [nidx, n]."""
    torch = _torch()
    out = torch.empty((idx.numel(), n), dtype=torch.float32, device=idx.device) if out is None else out
    _check(lib().b200_get_rows_q4_0(_ptr(table), _ptr(idx), _ptr(out), n, idx.numel(), vocab, _stream(idx.device)),
           "get_rows_q4_0")
    return out


def get_rows_q4_0_packed(w: "PackedWeight", idx, out=None):
    """GET_ROWS from a packed Q4_0 weight (rows of w.k elements) -> f32 [nidx, w.k]."""
    torch = _torch()
    out = torch.empty((idx.numel(), w.k), dtype=torch.float32, device=idx.device) if out is None else out
    _check(lib().b200_get_rows_q4_0_packed(_ptr(w.data), _ptr(idx), _ptr(out), w.k, idx.numel(), w.n,
                                           _stream(idx.device)), "get_rows_q4_0_packed")
    return out


class Upload:
    """set_tensor-style upload of one ggml weight into a packed copy:
    write(offset, host_bytes) in any order, from any thread; complete once
    every byte has arrived (the repack then has run)."""

    def __init__(self, wtype: int, n: int, k: int, device=None):
        torch = _torch()
        self.w = PackedWeight(wtype, n, k, torch.empty(packed_size(wtype, n, k), dtype=torch.uint8,
                                                       device=device or "cuda"))
        self.h = C.c_void_p()
        _check(lib().b200_upload_begin(wtype, n, k, _ptr(self.w.data), C.byref(self.h)), "b200_upload_begin")
        self.complete = False

    def write(self, offset: int, data: np.ndarray) -> bool:
        data = np.ascontiguousarray(data).view(np.uint8)
        done = C.c_int(0)
        _check(lib().b200_upload_write(self.h, offset, data.ctypes.data_as(C.c_void_p), data.nbytes, C.byref(done)),
               "b200_upload_write")
        self.complete = bool(done.value)
        return self.complete

    def close(self) -> int:
        if self.h:
            rc = lib().b200_upload_end(self.h)
            self.h = None
            return rc
        return OK


def swiglu(g, u, out=None):
    torch = _torch()
    out = torch.empty_like(g) if out is None else out
    _check(lib().b200_swiglu_f32(_ptr(g), _ptr(u), _ptr(out), g.numel(), _stream(g.device)), "swiglu")
    return out


def add(a, b, out=None):
    torch = _torch()
    out = torch.empty_like(a) if out is None else out
    _check(lib().b200_add_f32(_ptr(a), _ptr(b), _ptr(out), a.numel(), _stream(a.device)), "add")
    return out


def argmax(x):
    torch = _torch()
    out = torch.empty(1, dtype=torch.int32, device=x.device)
    _check(lib().b200_argmax_f32(_ptr(x), x.numel(), _ptr(out), _stream(x.device)), "argmax")
    return out


def kv_lengths_from_mask(mask_f16: np.ndarray) -> np.ndarray:
    m = np.ascontiguousarray(mask_f16, dtype=np.float16)
    if m.ndim == 1:
        m = m[None]
    out = np.empty(m.shape[0], dtype=np.int32)
    _check(
        lib().b200_kv_lengths_from_mask_f16(m.ctypes.data_as(C.c_void_p), m.shape[1], m.shape[0],
                                            out.ctypes.data_as(C.c_void_p)),
        "kv_lengths_from_mask",
    )
    return out
