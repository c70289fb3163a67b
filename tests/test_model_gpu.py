"""Whole-model decode parity (GPU): teacher-forced logits of every step vs the
CPU oracle on the same weights and KV cache, reduced depth, full or small
widths; greedy graph replay vs step-by-step decode."""
import numpy as np
import pytest

import oracle as O
from helpers import assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def build(cfg_kw, n_prefill, seed=11):
    import decode_model as M

    cfg = M.LlamaConfig(**cfg_kw)
    m = M.DecodeModel(cfg)
    m.init_synthetic(seed=seed, sigma=0.02)
    m.fill_kv_synthetic(seed=seed + 1, n_pos=n_prefill)
    kvd = cfg.n_head_kv * cfg.head_dim
    kc, vc = [], []
    for l in range(cfg.n_layer):
        k = np.zeros((cfg.kv_size, kvd), np.float16)
        v = np.zeros((cfg.kv_size, kvd), np.float16)
        k[:n_prefill] = m.export_kv(l, 0, n_prefill)
        v[:n_prefill] = m.export_kv(l, 1, n_prefill)
        kc.append(k)
        vc.append(v)
    ref = O.OracleLlama(cfg.as_dict(), M.oracle_weights(m), kc, vc)
    return m, ref


SMALL = dict(n_layer=2, d_model=512, n_head=8, n_head_kv=2, head_dim=64, d_ff=1024, vocab=2048, kv_size=96)


def test_small_teacher_forced_logits():
    m, ref = build(SMALL, n_prefill=40)
    toks = [3, 17, 1999, 0, 256, 1024, 7, 8]
    for i, t in enumerate(toks):
        pos = 40 + i
        nxt, logits = m.decode(t, pos, want_logits=True)
        r = ref.step(t, pos)
        assert_close(logits, ref.logits, what=f"step {i}")
        assert nxt == r or abs(ref.logits[nxt] - ref.logits[r]) <= 1e-3 * np.abs(ref.logits).max()
    m.close()


def test_llama70b_widths_two_layers():
    cfg = dict(n_layer=2, d_model=8192, n_head=64, n_head_kv=8, head_dim=128, d_ff=28672, vocab=128256,
               kv_size=4224)
    m, ref = build(cfg, n_prefill=4096)
    for i, t in enumerate([128000, 9906, 11]):
        pos = 4096 + i
        nxt, logits = m.decode(t, pos, want_logits=True)
        ref.step(t, pos)
        assert_close(logits, ref.logits, what=f"70b-width step {i}")
    m.close()


def test_graph_replay_greedy_matches_decode():
    import decode_model as M

    cfg = M.LlamaConfig(**SMALL)
    a = M.DecodeModel(cfg)
    a.init_synthetic(seed=5)
    a.fill_kv_synthetic(seed=6, n_pos=20)
    toks = []
    t = 42
    for i in range(6):
        t = a.decode(t, 20 + i)
        toks.append(t)
    b = M.DecodeModel(cfg)
    b.init_synthetic(seed=5)
    b.fill_kv_synthetic(seed=6, n_pos=20)
    b.capture()
    b.set_state(42, 20, advance=True)
    for _ in range(6):
        b.launch()
    torch.cuda.synchronize()
    # the last step's argmax is the last greedy token
    off, logits = b.logits()
    assert int(np.argmax(logits)) == toks[-1]
    prof = b.profile(iters=2)
    assert prof["qkv"] > 0 and prof["attn"] > 0 and prof["lm_head"] > 0
    a.close()
    b.close()


def test_model_rejects_bad_config():
    import b200_decode as B
    import decode_model as M

    bad = dict(SMALL)
    bad["n_head_kv"] = 3
    with pytest.raises(B.B200Error):
        M.DecodeModel(M.LlamaConfig(**bad))
    m = M.DecodeModel(M.LlamaConfig(**SMALL))
    m.init_synthetic(seed=1)
    with pytest.raises(B.B200Error):
        m.decode(0, SMALL["kv_size"])  # position past the cache
    with pytest.raises(B.B200Error):
        m.decode(SMALL["vocab"], 0)    # token id out of range
    m.close()
