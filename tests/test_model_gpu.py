"""Whole-model decode parity (GPU), reduced depth, small and full widths.

Every step is teacher-forced (the given token, not the model's own argmax)
and checked stage by stage (model_ref.stage_check): the oracle takes the
GPU's own input to each stage, every Q8_0 activation and per-block int32 dot
the step's GEMVs used must be bit-exact, and every fp stage -- roped q, K/V
rows, attention, both residuals, the SwiGLU output and the logits -- must be
within max relative error 1e-3, normwise and elementwise.

Without the stage forcing, logits drift further: two valid CPU accumulation
orders of the same semantics already differ by ~1e-2 after two layers,
because the Q8_0 activation quantisation is discontinuous
(test_accumulation_order_sensitivity_of_quantised_decode).  That drift is
measured below against the same CPU-vs-CPU figure, not held to 1e-3."""
import numpy as np
import pytest

import oracle as O
from helpers import TOL, errs
from model_ref import assert_stages, stage_check

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


def _free_run_drift_bound(cfg_kw, W, kc0, vc0, toks, pos0):
    """How far two valid CPU accumulation orders of the oracle drift apart
    over the same teacher-forced steps (max normwise error of the logits)."""
    worst = 0.0
    refs = []
    for mode in (0, 1):
        O.lib().ref_set_accum_mode(mode)
        r = O.OracleLlama(dict(cfg_kw, rope_theta=500000.0, rms_eps=1e-5), W, [k.copy() for k in kc0],
                          [v.copy() for v in vc0])
        out = []
        for i, t in enumerate(toks):
            r.step(t, pos0 + i)
            out.append(r.logits.copy())
        refs.append(out)
    O.lib().ref_set_accum_mode(0)
    for a, b in zip(*refs):
        worst = max(worst, errs(a, b)[0])
    return worst


def test_small_teacher_forced_per_stage():
    m, ref = build(SMALL, n_prefill=40)
    import decode_model as M

    cfg = M.LlamaConfig(**SMALL)
    W = M.oracle_weights(m)
    kc0 = [k.copy() for k in ref.k_cache]
    vc0 = [v.copy() for v in ref.v_cache]
    kc = [k.copy() for k in kc0]
    vc = [v.copy() for v in vc0]
    toks = [3, 17, 1999, 0, 256, 1024, 7, 8]
    drift = []
    for i, t in enumerate(toks):
        pos = 40 + i
        D = m.dump_step(t, pos)
        exact, fp = stage_check(cfg, W, kc, vc, D, t, pos)
        assert_stages(exact, fp, TOL, f"step {i}")
        ref.step(t, pos)
        drift.append(errs(D["logits"], ref.logits)[0])
    # free-running (no stage forcing): within a few times the CPU-vs-CPU drift
    cpu = _free_run_drift_bound(SMALL, W, kc0, vc0, toks, 40)
    assert max(drift) <= max(4 * cpu, 2 * TOL), (max(drift), cpu)
    m.close()


def test_llama70b_widths_two_layers_per_stage():
    import decode_model as M

    kw = dict(n_layer=2, d_model=8192, n_head=64, n_head_kv=8, head_dim=128, d_ff=28672, vocab=128256,
              kv_size=4224)
    m, ref = build(kw, n_prefill=4096)
    cfg = M.LlamaConfig(**kw)
    W = M.oracle_weights(m)
    kc = [k.copy() for k in ref.k_cache]
    vc = [v.copy() for v in ref.v_cache]
    for i, t in enumerate([128000, 9906]):
        pos = 4096 + i
        D = m.dump_step(t, pos)
        exact, fp = stage_check(cfg, W, kc, vc, D, t, pos)
        assert_stages(exact, fp, TOL, f"70b step {i}")
    m.close()


def test_dump_step_matches_debug_step_and_decode():
    """The full dump, the plain layer dump and the captured graph agree."""
    m, _ = build(SMALL, n_prefill=30)
    D = m.dump_step(9, 30)
    m2, _ = build(SMALL, n_prefill=30)
    x, q, a = m2.debug_step(9, 30)
    np.testing.assert_array_equal(D["x"], x)
    np.testing.assert_array_equal(D["q"], q)
    np.testing.assert_array_equal(D["att"], a)
    m3, _ = build(SMALL, n_prefill=30)
    _, logits = m3.decode(9, 30, want_logits=True)
    np.testing.assert_array_equal(D["logits"], logits)
    for mm in (m, m2, m3):
        mm.close()


def test_decode_matches_debug_step():
    """The captured graph and the eager layer-dump step produce the same logits."""
    m, _ = build(SMALL, n_prefill=30)
    nxt, logits = m.decode(9, 30, want_logits=True)
    m2, _ = build(SMALL, n_prefill=30)
    m2.debug_step(9, 30)
    _, l2 = m2.logits()
    np.testing.assert_array_equal(logits, l2)
    m.close()
    m2.close()


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
    assert b.time_gate_up(iters=2) > 0
    a.close()
    b.close()


FUSED_SHAPES = {
    # Llama-3-70B widths, two layers
    "llama70b_widths": dict(n_layer=2, d_model=8192, n_head=64, n_head_kv=8, head_dim=128, d_ff=28672,
                            vocab=128256, kv_size=4224),
    # 5632 / 148 CTAs: ~38 SwiGLU outputs per CTA, most 32-blocks shared by two CTAs
    "ff5632_d128": dict(n_layer=2, d_model=2048, n_head=16, n_head_kv=4, head_dim=128, d_ff=5632, vocab=4096,
                        kv_size=320),
    # head dim 64: attention slices of 16 blocks per kv head
    "d64": dict(n_layer=2, d_model=2048, n_head=32, n_head_kv=8, head_dim=64, d_ff=4096, vocab=4096,
                kv_size=320),
    # one rank's shapes of Llama-3-70B at tensor parallel 8: ~24 SwiGLU outputs per CTA (a 32-block can
    # span three CTAs) and an o projection of k = 1024 (the short-row GEMV path) fed by the image
    "tp8_rank": dict(n_layer=2, d_model=8192, n_head=8, n_head_kv=1, head_dim=128, d_ff=3584, vocab=4096,
                     kv_size=320),
}


@pytest.mark.parametrize("shape", list(FUSED_SHAPES))
def test_producer_quantised_activation_bit_identical(monkeypatch, shape):
    """The gate/up epilogue and the attention merge write the Q8_0 activation
    image that the down and o projections copy (B200_XQ_FUSED=1); with
    B200_XQ_FUSED=0 those GEMVs quantise f32 x in every CTA.  Same bytes, so
    every logit of every step is bit-identical."""
    import b200_decode as B
    import decode_model as M

    kw = FUSED_SHAPES[shape]
    n_pre = kw["kv_size"] - 128
    out = {}
    for fused in ("1", "0"):
        monkeypatch.setenv("B200_XQ_FUSED", fused)
        m = M.DecodeModel(M.LlamaConfig(**kw))
        m.init_synthetic(seed=21, sigma=0.02)
        m.fill_kv_synthetic(seed=22, n_pos=n_pre)
        t, steps = 7, []
        for i in range(3):
            t, logits = m.decode(t, n_pre + i, want_logits=True)
            steps.append((t, logits))
        out[fused] = steps
        m.close()
    for (t1, l1), (t0, l0) in zip(out["1"], out["0"]):
        assert t1 == t0
        np.testing.assert_array_equal(l1, l0)
    assert B.device_status() == 0


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


def test_synthetic_model_regenerates_bit_for_bit_on_host():
    """The device's synthetic weights and KV prefill equal the host
    generator's (oracle.synth_llama_weights / synth_llama_kv) byte for byte,
    so the CPU arm of bench.py times exactly the GPU arm's model."""
    import decode_model as M

    cfg = M.LlamaConfig(**SMALL)
    m = M.DecodeModel(cfg)
    m.init_synthetic(seed=11, sigma=0.02)
    m.fill_kv_synthetic(seed=12, n_pos=40)
    W = O.synth_llama_weights(cfg.as_dict(), 11, 0.02)
    G = M.oracle_weights(m)
    for key in ("tok_embd", "lm_head"):
        np.testing.assert_array_equal(G[key].reshape(-1), W[key].reshape(-1), err_msg=key)
    for key in ("wq", "wk", "wv", "wo", "wgate", "wup", "wdown"):
        for l in range(cfg.n_layer):
            np.testing.assert_array_equal(G[key][l].reshape(-1), W[key][l].reshape(-1), err_msg=f"{key}[{l}]")
    kc, vc = O.synth_llama_kv(cfg.as_dict(), 12, 40)
    for l in range(cfg.n_layer):
        np.testing.assert_array_equal(m.export_kv(l, 0, 40).view(np.uint16), kc[l][:40].view(np.uint16))
        np.testing.assert_array_equal(m.export_kv(l, 1, 40).view(np.uint16), vc[l][:40].view(np.uint16))
    m.close()


def test_step_timeline_adds_up():
    """b200_model_timeline: a captured step with device-clock stamps; the
    per-class advances add up to the step and every class ran."""
    import decode_model as M

    cfg = M.LlamaConfig(**SMALL)
    m = M.DecodeModel(cfg)
    m.init_synthetic(seed=5)
    m.fill_kv_synthetic(seed=6, n_pos=20)
    m.capture()
    m.set_state(42, 20, advance=True)
    m.timeline()
    tl = m.timeline()
    assert tl["step_us"] > 0
    adv = tl["advance_us"]
    assert abs(sum(adv.values()) - tl["step_us"]) <= 1e-3 * tl["step_us"] + 0.01
    for k in ("qkv", "attn", "o", "gate_up", "down", "lm_head"):
        assert tl["span_us"][k] > 0, k
        ph = tl["phases_us"][k]
        # marks in order inside the kernel, all within its span (the
        # earliest CTA no later than the latest one)
        assert 0.0 < ph["input_ready"] <= ph["exit"] + 1e-3, (k, ph)
        assert ph["first_chunk"] <= ph["exit"] + 1e-3 and ph["loop_done"] <= ph["exit"] + 1e-3, (k, ph)
        assert ph["input_ready_first_cta"] <= ph["input_ready"] + 1e-3, (k, ph)
        assert ph["loop_done_first_cta"] <= ph["loop_done"] + 1e-3, (k, ph)
        assert abs(ph["exit"] - tl["span_us"][k]) <= 0.01 + 1e-3 * tl["span_us"][k], (k, ph)
    assert adv["allreduce"] == 0.0  # one GPU: no all-reduce kernels
    import b200_decode as B

    assert B.device_status(reset=True) == 0
    m.close()
