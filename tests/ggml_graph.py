"""ctypes mirror of include/b200_graph.h and a builder for ggml-like decode
graphs (test helper).

``Graph`` creates b200_tensor descriptors the way ggml's graph builders lay
tensors out (ne[0] innermost, contiguous byte strides nb, views that share
data) and keeps them alive; ``llama_layer_graph`` builds one batch-1 Llama
decode layer with the ops, shapes and strides llama.cpp's graph uses
(RMS_NORM+MUL, three MUL_MATs, ROPE, SET_ROWS into the f16 cache, a permuted
q, FLASH_ATTN_EXT over strided cache views with a mask and the reference's
kv_lengths source, MUL_MAT, ADD, RMS_NORM+MUL, gate/up MUL_MATs, GLU
SWIGLU, MUL_MAT, ADD) plus the output norm, lm_head and ARGMAX.
"""
import ctypes as C
import struct

import numpy as np

F32, F16, Q4_0, Q8_0, I32, I64 = 0, 1, 2, 8, 26, 27
(OP_NONE, OP_VIEW, OP_GET_ROWS, OP_RMS_NORM, OP_MUL, OP_ADD, OP_MUL_MAT, OP_ROPE, OP_SET_ROWS,
 OP_FLASH_ATTN_EXT, OP_GLU, OP_ARGMAX, OP_CPY) = range(13)
GLU_SWIGLU = 2
TENSOR_WEIGHT = 1
CFG = dict(DISABLE_F16=1, DISABLE_Q4_0=2, DISABLE_Q8_0=4, DISABLE_FA=8, TRACE_SYNC=16, NVTX=32)

TYPE_SIZE = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), I32: (1, 4), I64: (1, 8)}


class Tensor(C.Structure):
    pass


Tensor._fields_ = [
    ("type", C.c_int), ("op", C.c_int), ("ne", C.c_int64 * 4), ("nb", C.c_size_t * 4),
    ("op_params", C.c_int32 * 16), ("src", C.POINTER(Tensor) * 10), ("data", C.c_void_p), ("extra", C.c_void_p),
    ("name", C.c_char_p), ("flags", C.c_uint),
]

_declared = False


def lib():
    global _declared
    import b200_decode as B

    L = B.lib()
    if not _declared:
        T = C.POINTER(Tensor)
        P = C.c_void_p
        sig = {
            "b200_nbytes": (C.c_size_t, [T]),
            "b200_config_flags": (C.c_uint, []),
            "b200_config_reload": (None, []),
            "b200_config_traces_op": (C.c_int, [C.c_int]),
            "b200_op_name": (C.c_char_p, [C.c_int]),
            "b200_supports_op": (C.c_int, [T]),
            "b200_is_matmul_weight": (C.c_int, [T, C.c_int]),
            "b200_alloc_size": (C.c_size_t, [T, C.c_int]),
            "b200_packed_offset": (C.c_size_t, [T]),
            "b200_buffer_alloc": (C.c_int, [C.c_int, C.c_size_t, C.c_int, C.POINTER(P)]),
            "b200_buffer_free": (None, [P]),
            "b200_buffer_base": (P, [P]),
            "b200_buffer_size": (C.c_size_t, [P]),
            "b200_buffer_init_tensor": (C.c_int, [P, T]),
            "b200_buffer_set_tensor": (C.c_int, [P, T, P, C.c_size_t, C.c_size_t]),
            "b200_buffer_get_tensor": (C.c_int, [P, T, P, C.c_size_t, C.c_size_t]),
            "b200_buffer_memset_tensor": (C.c_int, [P, T, C.c_uint8, C.c_size_t, C.c_size_t]),
            "b200_buffer_clear": (C.c_int, [P, C.c_uint8]),
            "b200_backend_create": (C.c_int, [C.c_int, C.POINTER(P)]),
            "b200_backend_free": (None, [P]),
            "b200_backend_stream": (P, [P]),
            "b200_backend_synchronize": (C.c_int, [P]),
            "b200_graph_compute": (C.c_int, [P, C.POINTER(T), C.c_int]),
            "b200_graph_failed_node": (C.c_int, [P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _declared = True
    return L


def f32_bits(v: float) -> int:
    return struct.unpack("<i", struct.pack("<f", v))[0]


def row_bytes(ttype, ne0):
    blck, size = TYPE_SIZE.get(ttype, (1, 1))
    return ne0 // blck * size


class Graph:
    """Descriptor factory: every tensor made here stays alive with the graph."""

    def __init__(self):
        self.keep = []
        self.nodes = []

    def tensor(self, ttype, ne, op=OP_NONE, src=(), params=(), name="", data=None, nb=None, node=None):
        t = Tensor()
        t.type = ttype
        t.op = op
        ne = list(ne) + [1] * (4 - len(ne))
        for i in range(4):
            t.ne[i] = ne[i]
        if nb is None:
            nb = [TYPE_SIZE.get(ttype, (1, 1))[1]]  # unknown types: descriptors for the rejection tests
            nb.append(row_bytes(ttype, ne[0]))
            nb.append(nb[1] * ne[1])
            nb.append(nb[2] * ne[2])
        for i in range(4):
            t.nb[i] = nb[i]
        for i, p in enumerate(params):
            t.op_params[i] = p
        for i, s in enumerate(src):
            if s is not None:
                t.src[i] = C.pointer(s)
        nm = name.encode()
        self.keep.append(nm)
        t.name = nm
        t.data = data
        self.keep.append(t)
        if node if node is not None else op != OP_NONE:
            self.nodes.append(t)
        return t

    def view(self, base, ne, nb, offset=0, name=""):
        return self.tensor(base.type, ne, op=OP_VIEW, src=(base,), name=name, data=base.data + offset, nb=nb)

    def node_array(self):
        arr = (C.POINTER(Tensor) * len(self.nodes))(*[C.pointer(t) for t in self.nodes])
        self.keep.append(arr)
        return arr, len(self.nodes)


def nbytes(t) -> int:
    return int(lib().b200_nbytes(C.byref(t)))


def supports(t) -> bool:
    return lib().b200_supports_op(C.byref(t)) == 1


def rope_params(n_dims, freq_base, mode=0, freq_scale=1.0, ext_factor=0.0, attn_factor=1.0):
    """ggml_rope_impl's op_params: n_past, n_dims, mode, n_ctx, n_ctx_orig,
    then freq_base, freq_scale, ext_factor, attn_factor, beta_fast, beta_slow."""
    return [0, n_dims, mode, 0, 0, f32_bits(freq_base), f32_bits(freq_scale), f32_bits(ext_factor),
            f32_bits(attn_factor), f32_bits(32.0), f32_bits(1.0)]


def fa_params(scale, max_bias=0.0, softcap=0.0):
    return [f32_bits(scale), f32_bits(max_bias), f32_bits(softcap), 0]


def np_f16_bits(a):
    return np.ascontiguousarray(a, dtype=np.float16).view(np.uint16)
