"""The ggml-backend core on the GPU: one Llama decode layer (plus the
output norm, the tied lm_head and ARGMAX) built as a descriptor graph with
llama.cpp's ops, shapes and strides, run by b200_graph_compute, and every
node checked against the CPU oracle fed that node's GPU inputs.

Weights live in a b200 weight buffer and arrive through set_tensor in
shuffled chunks, as ggml's model loader may send them; the buffer keeps the
ggml bytes at tensor->data (GET_ROWS of the tied embedding reads them,
get_tensor returns them) and the packed copy behind them (MUL_MAT reads it).
"""
import ctypes as C

import numpy as np
import pytest

import ggml_graph as G
import oracle as O
from helpers import TOL, assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

CFG = dict(d=1024, hq=8, hkv=2, D=128, ff=2048, vocab=4096, kv=512, theta=500000.0, eps=1e-5)


class Buf:
    def __init__(self, size, weights):
        self.h = C.c_void_p()
        rc = G.lib().b200_buffer_alloc(0, size, 1 if weights else 0, C.byref(self.h))
        assert rc == 0, rc
        self.base = G.lib().b200_buffer_base(self.h)
        self.off = 0

    def place(self, t, weights):
        t.data = self.base + self.off
        self.off += (G.lib().b200_alloc_size(C.byref(t), 1 if weights else 0) + 255) // 256 * 256
        assert G.lib().b200_buffer_init_tensor(self.h, C.byref(t)) == 0

    def set(self, t, host: np.ndarray, chunks=1, rng=None):
        raw = np.ascontiguousarray(host).view(np.uint8).reshape(-1)
        cuts = sorted(set([0, raw.size] + (list(rng.integers(1, raw.size, chunks - 1)) if chunks > 1 else [])))
        pieces = list(zip(cuts[:-1], cuts[1:]))
        if rng is not None:
            rng.shuffle(pieces)
        for a, b in pieces:
            chunk = np.ascontiguousarray(raw[a:b])
            rc = G.lib().b200_buffer_set_tensor(self.h, C.byref(t), chunk.ctypes.data_as(C.c_void_p), int(a),
                                               int(b - a))
            assert rc == 0, rc

    def get(self, t, nbytes):
        out = np.empty(nbytes, np.uint8)
        assert G.lib().b200_buffer_get_tensor(self.h, C.byref(t), out.ctypes.data_as(C.c_void_p), 0, nbytes) == 0
        return out

    def free(self):
        G.lib().b200_buffer_free(self.h)


def _dev(t):
    return int(t.data_ptr())


def build_layer(rng):
    c = CFG
    d, hq, hkv, D, ff, vocab, kv = c["d"], c["hq"], c["hkv"], c["D"], c["ff"], c["vocab"], c["kv"]
    qd, kvd = hq * D, hkv * D
    W = {
        "tok_embd": O.synth_q4_0(101, 0.02, 0, vocab, d), "wq": O.synth_q4_0(102, 0.02, 0, qd, d),
        "wk": O.synth_q4_0(103, 0.02, 0, kvd, d), "wv": O.synth_q4_0(104, 0.02, 0, kvd, d),
        "wo": O.synth_q4_0(105, 0.02, 0, d, qd), "wgate": O.synth_q4_0(106, 0.02, 0, ff, d),
        "wup": O.synth_q4_0(107, 0.02, 0, ff, d), "wdown": O.synth_q4_0(108, 0.02, 0, d, ff),
    }
    norms = {k: (1 + 0.1 * rng.standard_normal(d)).astype(np.float32) for k in ("attn_norm", "ffn_norm", "out_norm")}
    g = G.Graph()
    shapes = {"tok_embd": (d, vocab), "wq": (d, qd), "wk": (d, kvd), "wv": (d, kvd), "wo": (qd, d), "wgate": (d, ff),
              "wup": (d, ff), "wdown": (ff, d)}
    wt = {k: g.tensor(G.Q4_0, shapes[k], name=k + ".weight") for k in shapes}
    size = sum((G.lib().b200_alloc_size(C.byref(t), 1) + 255) // 256 * 256 for t in wt.values())
    wb = Buf(size, True)
    for k, t in wt.items():
        wb.place(t, True)
        wb.set(t, W[k], chunks=5, rng=rng)
    T = {}  # device memory of activations, inputs and caches (torch)

    def act(name, ttype, ne, **kw):
        dt = {G.F32: torch.float32, G.F16: torch.float16, G.I32: torch.int32, G.I64: torch.int64}[ttype]
        assert name not in T, name
        n = int(np.prod(ne))
        T[name] = torch.zeros(n, dtype=dt, device="cuda")
        return g.tensor(ttype, ne, data=_dev(T[name]), name=name, node=False, **kw)

    tokens = act("tokens", G.I32, [1])
    pos = act("pos", G.I32, [1])
    kv_idx = act("kv_idx", G.I64, [1])
    kv_len = act("kv_len", G.I32, [1])
    mask = act("mask", G.F16, [kv, 64])
    kcache = act("k_cache", G.F16, [kvd, kv])
    vcache = act("v_cache", G.F16, [kvd, kv])
    nt = {k: act(k + ".weight", G.F32, [d]) for k in norms}
    for k in norms:
        T[k + ".weight"].copy_(torch.from_numpy(norms[k]))

    def node(name, ttype, ne, op, src, params=()):
        assert name not in T, name  # every descriptor keeps its own device memory alive
        dt = {G.F32: torch.float32, G.I32: torch.int32}[ttype]
        T[name] = torch.full((int(np.prod(ne)),), float("nan") if ttype == G.F32 else -1, dtype=dt, device="cuda")
        return g.tensor(ttype, ne, op=op, src=src, params=params, data=_dev(T[name]), name=name)

    eps = [G.f32_bits(c["eps"])]
    inp = node("inp_embd", G.F32, [d, 1], G.OP_GET_ROWS, (wt["tok_embd"], tokens))
    rn = node("attn_rms", G.F32, [d, 1], G.OP_RMS_NORM, (inp,), eps)
    cur = node("attn_norm", G.F32, [d, 1], G.OP_MUL, (rn, nt["attn_norm"]))
    q = node("Qcur", G.F32, [qd, 1], G.OP_MUL_MAT, (wt["wq"], cur))
    k = node("Kcur", G.F32, [kvd, 1], G.OP_MUL_MAT, (wt["wk"], cur))
    v = node("Vcur", G.F32, [kvd, 1], G.OP_MUL_MAT, (wt["wv"], cur))
    q3 = g.view(q, [D, hq, 1], [4, D * 4, qd * 4, qd * 4], name="Qcur_3d")
    k3 = g.view(k, [D, hkv, 1], [4, D * 4, kvd * 4, kvd * 4], name="Kcur_3d")
    rp = G.rope_params(D, c["theta"])
    qr = node("Qrope", G.F32, [D, hq, 1], G.OP_ROPE, (q3, pos), rp)
    kr = node("Krope", G.F32, [D, hkv, 1], G.OP_ROPE, (k3, pos), rp)
    kr2 = g.view(kr, [kvd, 1], [4, kvd * 4, kvd * 4, kvd * 4], name="Krope_2d")
    g.tensor(G.F16, [kvd, kv], op=G.OP_SET_ROWS, src=(kr2, kv_idx), data=kcache.data, nb=list(kcache.nb),
             name="k_cache_set")
    g.tensor(G.F16, [kvd, kv], op=G.OP_SET_ROWS, src=(v, kv_idx), data=vcache.data, nb=list(vcache.nb),
             name="v_cache_set")
    qp = g.view(qr, [D, 1, hq], [4, qd * 4, D * 4, qd * 4], name="q_perm")
    kview = g.view(kcache, [D, kv, hkv], [2, kvd * 2, D * 2, kvd * 2 * kv], name="k_view")
    vview = g.view(vcache, [D, kv, hkv], [2, kvd * 2, D * 2, kvd * 2 * kv], name="v_view")
    fa = node("fattn", G.F32, [D, hq, 1], G.OP_FLASH_ATTN_EXT, (qp, kview, vview, mask, None, kv_len),
              G.fa_params(D ** -0.5))
    fa2 = g.view(fa, [qd, 1], [4, qd * 4, qd * 4, qd * 4], name="fattn_2d")
    o = node("attn_out", G.F32, [d, 1], G.OP_MUL_MAT, (wt["wo"], fa2))
    ffn_inp = node("ffn_inp", G.F32, [d, 1], G.OP_ADD, (o, inp))
    rn2 = node("ffn_rms", G.F32, [d, 1], G.OP_RMS_NORM, (ffn_inp,), eps)
    cur2 = node("ffn_norm", G.F32, [d, 1], G.OP_MUL, (rn2, nt["ffn_norm"]))
    gate = node("ffn_gate", G.F32, [ff, 1], G.OP_MUL_MAT, (wt["wgate"], cur2))
    up = node("ffn_up", G.F32, [ff, 1], G.OP_MUL_MAT, (wt["wup"], cur2))
    h = node("ffn_swiglu", G.F32, [ff, 1], G.OP_GLU, (gate, up), [G.GLU_SWIGLU, 0])
    dn = node("ffn_down", G.F32, [d, 1], G.OP_MUL_MAT, (wt["wdown"], h))
    out = node("l_out", G.F32, [d, 1], G.OP_ADD, (dn, ffn_inp))
    rn3 = node("out_rms", G.F32, [d, 1], G.OP_RMS_NORM, (out,), eps)
    cur3 = node("result_norm", G.F32, [d, 1], G.OP_MUL, (rn3, nt["out_norm"]))
    node("result_output", G.F32, [vocab, 1], G.OP_MUL_MAT, (wt["tok_embd"], cur3))
    node("argmax", G.I32, [1], G.OP_ARGMAX, (g.nodes[-1],))
    return g, W, norms, T, wb, wt


def _np(T, name, dtype=np.float32):
    return T[name].cpu().numpy().astype(dtype, copy=False)


def _run_step(be, g, T, tok, p, prefill):
    c = CFG
    T["tokens"].fill_(tok)
    T["pos"].fill_(p)
    T["kv_idx"].fill_(p)
    T["kv_len"].fill_(p + 1)
    m = np.zeros((64, c["kv"]), np.float16)
    m[:, p + 1:] = -np.inf
    T["mask"].copy_(torch.from_numpy(m.reshape(-1)))
    torch.cuda.synchronize()
    arr, n = g.node_array()
    rc = G.lib().b200_graph_compute(be, arr, n)
    assert rc == 0, (rc, G.lib().b200_graph_failed_node(be))
    assert G.lib().b200_backend_synchronize(be) == 0


def _check_step(W, norms, T, tok, p):
    """Every node against the oracle fed the GPU's inputs of that node."""
    c = CFG
    d, hq, hkv, D, vocab = c["d"], c["hq"], c["hkv"], c["D"], c["vocab"]
    kvd = hkv * D
    inp = _np(T, "inp_embd")
    np.testing.assert_array_equal(inp, O.dequantize_q4_0(W["tok_embd"][tok].copy()))
    cur = _np(T, "attn_norm")
    np.testing.assert_array_equal(cur, O.rms_norm_mul(inp, norms["attn_norm"], c["eps"]))
    for name, w in (("Qcur", "wq"), ("Kcur", "wk"), ("Vcur", "wv")):
        assert_close(_np(T, name), O.mul_mat_q4_0(W[w], cur), TOL, name)
    assert_close(_np(T, "Qrope"), O.rope_norm(_np(T, "Qcur"), hq, D, p, c["theta"]), TOL, "Qrope")
    kr = O.rope_norm(_np(T, "Kcur"), hkv, D, p, c["theta"])
    assert_close(_np(T, "Krope"), kr, TOL, "Krope")
    kc = _np(T, "k_cache", np.float16).reshape(c["kv"], kvd)
    vc = _np(T, "v_cache", np.float16).reshape(c["kv"], kvd)
    np.testing.assert_array_equal(kc[p].view(np.uint16), _np(T, "Krope").astype(np.float16).view(np.uint16))
    np.testing.assert_array_equal(vc[p].view(np.uint16), _np(T, "Vcur").astype(np.float16).view(np.uint16))
    att = O.flash_attn_decode(_np(T, "Qrope").reshape(hq, D), kc.reshape(-1, hkv, D), vc.reshape(-1, hkv, D),
                              _np(T, "mask", np.float16)[:c["kv"]], kv_len=p + 1)
    assert_close(_np(T, "fattn"), att.reshape(-1), TOL, "fattn")
    assert_close(_np(T, "attn_out"), O.mul_mat_q4_0(W["wo"], _np(T, "fattn")), TOL, "attn_out")
    np.testing.assert_array_equal(_np(T, "ffn_inp"), _np(T, "attn_out") + inp)
    cur2 = _np(T, "ffn_norm")
    np.testing.assert_array_equal(cur2, O.rms_norm_mul(_np(T, "ffn_inp"), norms["ffn_norm"], c["eps"]))
    gte, up = _np(T, "ffn_gate"), _np(T, "ffn_up")
    assert_close(gte, O.mul_mat_q4_0(W["wgate"], cur2), TOL, "ffn_gate")
    assert_close(up, O.mul_mat_q4_0(W["wup"], cur2), TOL, "ffn_up")
    assert_close(_np(T, "ffn_swiglu"), (gte / (1 + np.exp(-gte.astype(np.float64)))) * up, TOL, "swiglu")
    assert_close(_np(T, "ffn_down"), O.mul_mat_q4_0(W["wdown"], _np(T, "ffn_swiglu")), TOL, "ffn_down")
    np.testing.assert_array_equal(_np(T, "l_out"), _np(T, "ffn_down") + _np(T, "ffn_inp"))
    cur3 = _np(T, "result_norm")
    np.testing.assert_array_equal(cur3, O.rms_norm_mul(_np(T, "l_out"), norms["out_norm"], c["eps"]))
    logits = _np(T, "result_output")
    assert logits.shape == (vocab,)
    assert_close(logits, O.mul_mat_q4_0(W["tok_embd"], cur3), TOL, "logits")
    assert int(T["argmax"].item()) == int(np.argmax(logits))


def test_llama_layer_descriptor_graph_matches_oracle():
    import b200_decode as B

    rng = np.random.default_rng(2)
    g, W, norms, T, wb, wt = build_layer(rng)
    # KV cache prefill (positions < 300)
    p0 = 300
    kvd = CFG["hkv"] * CFG["D"]
    pre = rng.standard_normal((CFG["kv"], kvd)).astype(np.float16)
    pre[p0:] = 0
    T["k_cache"].copy_(torch.from_numpy(pre.reshape(-1)))
    T["v_cache"].copy_(torch.from_numpy(rng.standard_normal((CFG["kv"], kvd)).astype(np.float16).reshape(-1)))
    be = C.c_void_p()
    assert G.lib().b200_backend_create(0, C.byref(be)) == 0
    try:
        for i, tok in enumerate([17, 4000, 1]):
            _run_step(be, g, T, tok, p0 + i, p0)
            _check_step(W, norms, T, tok, p0 + i)
        # get_tensor returns the ggml bytes of a packed weight (the dual layout keeps them)
        for k in ("tok_embd", "wdown"):
            got = wb.get(wt[k], W[k].size)
            np.testing.assert_array_equal(got, W[k].reshape(-1))
            assert wt[k].flags & G.TENSOR_WEIGHT and wt[k].extra == wt[k].data + G.lib().b200_packed_offset(
                C.byref(wt[k]))
        assert B.device_status(reset=True) == 0
    finally:
        G.lib().b200_backend_free(be)
        wb.free()


def test_graph_trace_sync_and_unsupported_node(monkeypatch, capfd):
    """GGML_B200_TRACE_SYNC logs every node's begin/end and synchronises; a
    node supports_op refuses stops the graph with EUNSUPPORTED and its
    index."""
    rng = np.random.default_rng(3)
    g, W, norms, T, wb, wt = build_layer(rng)
    be = C.c_void_p()
    assert G.lib().b200_backend_create(0, C.byref(be)) == 0
    try:
        monkeypatch.setenv("GGML_B200_TRACE_SYNC", "MUL_MAT,FLASH_ATTN_EXT")
        G.lib().b200_config_reload()
        _run_step(be, g, T, 5, 10, 0)
        err = capfd.readouterr().err
        assert "[b200] node" in err and "MUL_MAT Qcur: begin" in err and "FLASH_ATTN_EXT fattn: end" in err
        assert "ROPE" not in err
        monkeypatch.setenv("GGML_B200_DISABLE_FA", "1")
        G.lib().b200_config_reload()
        arr, n = g.node_array()
        assert G.lib().b200_graph_compute(be, arr, n) == -3
        failed = G.lib().b200_graph_failed_node(be)
        assert g.nodes[failed].op == G.OP_FLASH_ATTN_EXT
    finally:
        monkeypatch.delenv("GGML_B200_TRACE_SYNC", raising=False)
        monkeypatch.delenv("GGML_B200_DISABLE_FA", raising=False)
        G.lib().b200_config_reload()
        G.lib().b200_backend_free(be)
        wb.free()


@pytest.mark.parametrize("wtype,m", [(G.F16, 1), (G.F16, 4), (G.F16, 33), (G.Q4_0, 1), (G.Q4_0, 3), (G.Q8_0, 2)])
def test_graph_mul_mat_columns(wtype, m):
    """MUL_MAT nodes with several src1 columns: F16 M <= 8 on the small-M
    kernel, M > 8 on the tcgen05 prefill GEMM, Q4_0 / Q8_0 column by column;
    weights through the buffer's set_tensor (packed copy) as in the model."""
    n, k = 384, 1024
    r = np.random.default_rng(40 + m + wtype)
    if wtype == G.F16:
        wh = (r.standard_normal((n, k)) * 0.02).astype(np.float16)
        ref_fn = lambda xj: O.mul_mat_f16(wh, xj)  # noqa: E731
    elif wtype == G.Q4_0:
        wh = O.synth_q4_0(77, 0.02, 0, n, k)
        ref_fn = lambda xj: O.mul_mat_q4_0(wh, xj)  # noqa: E731
    else:
        wh = O.quantize_q8_0((r.standard_normal((n, k)) * 0.02).astype(np.float32))
        ref_fn = lambda xj: O.mul_mat_q8_0(wh, xj)  # noqa: E731
    g = G.Graph()
    w = g.tensor(wtype, [k, n], name="blk.0.attn_q.weight")
    wb = Buf((G.lib().b200_alloc_size(C.byref(w), 1) + 255) // 256 * 256, True)
    wb.place(w, True)
    wb.set(w, wh)
    x = r.standard_normal((m, k)).astype(np.float32)
    tx = torch.from_numpy(x).cuda()
    ty = torch.full((m, n), float("nan"), device="cuda")
    xt = g.tensor(G.F32, [k, m], data=_dev(tx), node=False, name="x")
    g.tensor(G.F32, [n, m], op=G.OP_MUL_MAT, src=(w, xt), data=_dev(ty), name="y")
    be = C.c_void_p()
    assert G.lib().b200_backend_create(0, C.byref(be)) == 0
    try:
        arr, cnt = g.node_array()
        assert G.lib().b200_graph_compute(be, arr, cnt) == 0
        assert G.lib().b200_backend_synchronize(be) == 0
        y = ty.cpu().numpy()
        for j in range(m):
            assert_close(y[j], ref_fn(x[j]), TOL, f"type {wtype} column {j} of {m}")
    finally:
        G.lib().b200_backend_free(be)
        wb.free()
