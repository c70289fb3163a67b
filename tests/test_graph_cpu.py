"""The ggml-backend core on the host (no GPU): supports_op decisions on the
reference's edge cases, get_alloc_size of the dual ggml + packed weight
layout, ggml_nbytes of strided views, and the environment registry
(GGML_B200_DISABLE_*, GGML_B200_TRACE_SYNC).  The reference's own gate is
supports_op in patch:1925-1986 (FLASH_ATTN_EXT: patch:1964-1983)."""
import numpy as np
import pytest

import ggml_graph as G

FAKE = 1 << 20  # descriptors only: supports_op and sizes never touch data


@pytest.fixture(autouse=True)
def _fresh_config(monkeypatch):
    for k in ("GGML_B200_DISABLE_F16", "GGML_B200_DISABLE_Q4_0", "GGML_B200_DISABLE_Q8_0", "GGML_B200_DISABLE_FA",
              "GGML_B200_TRACE_SYNC", "GGML_B200_NVTX"):
        monkeypatch.delenv(k, raising=False)
    G.lib().b200_config_reload()
    yield
    monkeypatch.undo()
    G.lib().b200_config_reload()


def _fa(g, D=128, hq=12, hkv=2, n_kv=4096, qtype=G.F32, ktype=G.F16, mask=True, n_tok=1, params=None,
        kv_len=False, sinks=False, nb_pad=0):
    q = g.tensor(qtype, [D, n_tok, hq], data=FAKE, nb=[4, hq * D * 4, D * 4, hq * D * 4 * n_tok])
    esz = 2 if ktype == G.F16 else 4
    kvd = hkv * D
    k = g.tensor(ktype, [D, n_kv, hkv], data=FAKE, nb=[esz, kvd * esz + nb_pad, D * esz, kvd * esz * n_kv])
    v = g.tensor(ktype, [D, n_kv, hkv], data=FAKE, nb=[esz, kvd * esz + nb_pad, D * esz, kvd * esz * n_kv])
    m = g.tensor(G.F16, [n_kv, 64], data=FAKE) if mask else None
    s = g.tensor(G.F32, [hq], data=FAKE) if sinks else None
    kl = g.tensor(G.I32, [1], data=FAKE) if kv_len else None
    return g.tensor(G.F32, [D, hq, n_tok], op=G.OP_FLASH_ATTN_EXT, src=(q, k, v, m, s, kl),
                    params=params if params is not None else G.fa_params(D ** -0.5), data=FAKE)


def test_fa_gate_accepts_decode_shapes():
    g = G.Graph()
    for D, hq, hkv in ((64, 14, 2), (128, 12, 2), (128, 64, 8), (256, 16, 4), (128, 8, 8)):
        assert G.supports(_fa(g, D=D, hq=hq, hkv=hkv)), (D, hq, hkv)
    assert G.supports(_fa(g, mask=False))
    assert G.supports(_fa(g, kv_len=True))  # src[5] kv_lengths (patch:2009-2023)


@pytest.mark.parametrize("what", ["head_dim_96", "two_tokens", "f32_kv", "f16_q", "alibi", "softcap", "sinks",
                                  "gqa_ratio", "unaligned_rows"])
def test_fa_gate_rejects(what):
    g = G.Graph()
    kw = {
        "head_dim_96": dict(D=96), "two_tokens": dict(n_tok=2), "f32_kv": dict(ktype=G.F32),
        "f16_q": dict(qtype=G.F16), "alibi": dict(params=G.fa_params(0.1, max_bias=8.0)),
        "softcap": dict(params=G.fa_params(0.1, softcap=30.0)), "sinks": dict(sinks=True),
        "gqa_ratio": dict(hq=12, hkv=5), "unaligned_rows": dict(nb_pad=2),
    }[what]
    assert not G.supports(_fa(g, **kw))


def _mm(g, wtype, n=256, k=512, m=1, w3d=False):
    w = g.tensor(wtype, [k, n, 2 if w3d else 1], data=FAKE)
    x = g.tensor(G.F32, [k, m], data=FAKE)
    return g.tensor(G.F32, [n, m], op=G.OP_MUL_MAT, src=(w, x), data=FAKE)


def test_mul_mat_gate():
    g = G.Graph()
    for t in (G.F16, G.Q4_0, G.Q8_0):
        assert G.supports(_mm(g, t))
        assert G.supports(_mm(g, t, m=4))
        assert G.supports(_mm(g, t, m=33))  # prefill columns run here too (no CPU fallback)
    assert not G.supports(_mm(g, 3))  # Q4_1
    assert not G.supports(_mm(g, G.Q4_0, w3d=True))
    assert not G.supports(_mm(g, G.Q4_0, k=500))  # not a whole number of blocks


@pytest.mark.parametrize("var,wtype", [("GGML_B200_DISABLE_F16", G.F16), ("GGML_B200_DISABLE_Q4_0", G.Q4_0),
                                       ("GGML_B200_DISABLE_Q8_0", G.Q8_0)])
def test_disable_switches_refuse_their_type_only(monkeypatch, var, wtype):
    g = G.Graph()
    monkeypatch.setenv(var, "1")
    G.lib().b200_config_reload()
    assert not G.supports(_mm(g, wtype))
    others = [t for t in (G.F16, G.Q4_0, G.Q8_0) if t != wtype]
    assert all(G.supports(_mm(g, t)) for t in others)
    assert G.supports(_fa(g))


def test_disable_fa(monkeypatch):
    g = G.Graph()
    monkeypatch.setenv("GGML_B200_DISABLE_FA", "1")
    G.lib().b200_config_reload()
    assert G.lib().b200_config_flags() & G.CFG["DISABLE_FA"]
    assert not G.supports(_fa(g))
    assert G.supports(_mm(g, G.Q4_0))


def test_trace_sync_registry(monkeypatch):
    L = G.lib()
    monkeypatch.setenv("GGML_B200_TRACE_SYNC", "MUL_MAT,ROPE")
    L.b200_config_reload()
    assert L.b200_config_flags() & G.CFG["TRACE_SYNC"]
    assert L.b200_config_traces_op(G.OP_MUL_MAT) and L.b200_config_traces_op(G.OP_ROPE)
    assert not L.b200_config_traces_op(G.OP_FLASH_ATTN_EXT)
    monkeypatch.setenv("GGML_B200_TRACE_SYNC", "1")
    L.b200_config_reload()
    assert all(L.b200_config_traces_op(op) for op in range(13))
    monkeypatch.setenv("GGML_B200_TRACE_SYNC", "0")
    L.b200_config_reload()
    assert not L.b200_config_flags() & G.CFG["TRACE_SYNC"]
    assert L.b200_op_name(G.OP_FLASH_ATTN_EXT) == b"FLASH_ATTN_EXT"


def test_neighbour_op_gates():
    g = G.Graph()
    x = g.tensor(G.F32, [512, 1], data=FAKE)
    w = g.tensor(G.F32, [512], data=FAKE)
    rn = g.tensor(G.F32, [512, 1], op=G.OP_RMS_NORM, src=(x,), params=[G.f32_bits(1e-5)], data=FAKE)
    assert G.supports(rn)
    assert G.supports(g.tensor(G.F32, [512, 1], op=G.OP_MUL, src=(rn, w), data=FAKE))
    assert not G.supports(g.tensor(G.F32, [512, 1], op=G.OP_MUL, src=(rn, g.tensor(G.F32, [256], data=FAKE)),
                                   data=FAKE))
    q = g.tensor(G.F32, [128, 8, 1], data=FAKE)
    pos = g.tensor(G.I32, [1], data=FAKE)
    assert G.supports(g.tensor(G.F32, [128, 8, 1], op=G.OP_ROPE, src=(q, pos), params=G.rope_params(128, 5e5),
                               data=FAKE))
    # NEOX mode, partial rotation, YaRN scaling: not on this path
    for p in (G.rope_params(128, 5e5, mode=2), G.rope_params(64, 5e5), G.rope_params(128, 5e5, freq_scale=0.25)):
        assert not G.supports(g.tensor(G.F32, [128, 8, 1], op=G.OP_ROPE, src=(q, pos), params=p, data=FAKE))
    a = g.tensor(G.F32, [1024], data=FAKE)
    b = g.tensor(G.F32, [1024], data=FAKE)
    assert G.supports(g.tensor(G.F32, [1024], op=G.OP_GLU, src=(a, b), params=[G.GLU_SWIGLU, 0], data=FAKE))
    assert not G.supports(g.tensor(G.F32, [1024], op=G.OP_GLU, src=(a, b), params=[1, 0], data=FAKE))  # GEGLU
    cache = g.tensor(G.F16, [1024, 4096], data=FAKE)
    rows = g.tensor(G.F32, [1024, 1], data=FAKE)
    idx = g.tensor(G.I64, [1], data=FAKE)
    assert G.supports(g.tensor(G.F16, [1024, 4096], op=G.OP_SET_ROWS, src=(rows, idx), data=FAKE,
                               nb=list(cache.nb)))
    assert not G.supports(g.tensor(G.F16, [1024, 4096], op=G.OP_SET_ROWS, src=(rows, pos), data=FAKE,
                                   nb=list(cache.nb)))  # I32 row ids
    tab = g.tensor(G.Q4_0, [512, 2048], data=FAKE)
    tok = g.tensor(G.I32, [3], data=FAKE)
    assert G.supports(g.tensor(G.F32, [512, 3], op=G.OP_GET_ROWS, src=(tab, tok), data=FAKE))
    assert not G.supports(g.tensor(G.F32, [512, 3], op=G.OP_GET_ROWS, src=(g.tensor(G.F16, [512, 2048], data=FAKE),
                                                                           tok), data=FAKE))


def test_alloc_size_dual_layout_and_nbytes():
    import b200_decode as B

    L = G.lib()
    g = G.Graph()
    for wtype, n, k in ((G.Q4_0, 1536, 8960), (G.Q8_0, 151936, 1536), (G.F16, 8960, 1536)):
        w = g.tensor(wtype, [k, n], data=FAKE, name="blk.0.ffn_down.weight")
        # the same tensor under a cache's name is never packed (a 2-D f16 KV cache shares the buffer)
        assert L.b200_is_matmul_weight(g.tensor(wtype, [k, n], data=FAKE, name="cache_k_l0"), 1) == 0
        nb = G.nbytes(w)
        assert nb == n * G.row_bytes(wtype, k)
        assert L.b200_is_matmul_weight(w, 1) == 1 and L.b200_is_matmul_weight(w, 0) == 0
        off = L.b200_packed_offset(w)
        assert off % 256 == 0 and off >= nb and off - nb < 256
        assert L.b200_alloc_size(w, 1) == off + B.packed_size(wtype, n, k)
        assert L.b200_alloc_size(w, 0) == nb
    # activations, caches and ids are never packed
    for t in (g.tensor(G.F32, [4096, 1], data=FAKE), g.tensor(G.I32, [7], data=FAKE)):
        assert L.b200_alloc_size(t, 1) == G.nbytes(t)
    # a strided view: ggml_nbytes = row + sum (ne[i] - 1) nb[i]
    v = g.tensor(G.F16, [128, 4096, 8], data=FAKE, nb=[2, 8 * 128 * 2, 128 * 2, 8 * 128 * 2 * 4096])
    assert G.nbytes(v) == 2 + 127 * 2 + 4095 * 2048 + 7 * 256
    assert G.nbytes(g.tensor(17, [32], data=FAKE)) == 0  # unknown type
