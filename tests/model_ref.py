"""Stage-level teacher forcing for whole-model parity (test helper).

Q8_0 activation quantisation is discontinuous: an ulp of difference in an
fp32 sum (two valid accumulation orders) can flip one int8 of an activation
block, and a flipped int8 moves the next GEMV's outputs by ~1e-4 of their
range, far beyond an elementwise 1e-3 bar on outputs near zero.  The check
therefore feeds the oracle, stage by stage, the GPU's own input to that
stage (from b200_model_debug_step_ex) and asks of every stage:

* integer stages bit-exact: each Q8_0 activation the GPU's GEMVs consumed
  equals the oracle's quantisation of the GPU's f32 stage input (RMSNorm
  output for QKV / gate-up / lm_head, attention output for O, SwiGLU output
  for down), and every per-(row, 32-block) int32 dot equals the oracle's dot
  of the same weight block with those activation bytes;
* fp stages (roped q, K/V rows, attention, residual after O, SwiGLU output,
  residual after down, logits) within max relative error 1e-3, both
  normwise and elementwise (helpers.errs), against the oracle run from the
  same Q8_0 bytes.
"""
import numpy as np

import oracle as O
from helpers import errs

QB = 34  # bytes of a ggml block_q8_0


def _rows(w, nrows):
    return np.ascontiguousarray(w).reshape(nrows, -1)


def _mismatch(a, b):
    a = np.asarray(a)
    b = np.asarray(b)
    return int(np.count_nonzero(a != b)) if a.shape == b.shape else -1


def stage_check(cfg, W, kc, vc, D, tok, pos):
    """Checks one dumped step.  cfg: LlamaConfig; W: oracle weights (ggml
    layouts, tp_world 1); kc/vc: the oracle's KV caches, which receive the
    GPU's K/V rows at pos; D: DecodeModel.dump_step(...) of (tok, pos).
    Returns (exact, fp): exact maps a name to its number of mismatching
    entries (0 = bit-exact), fp maps a stage to (normwise, elementwise)."""
    d, Dh, hq, hkv, ff = cfg.d_model, cfg.head_dim, cfg.n_head, cfg.n_head_kv, cfg.d_ff
    qd, kvd = hq * Dh, hkv * Dh
    exact, fp = {}, {}
    emb = O.dequantize_q4_0(_rows(W["tok_embd"], cfg.vocab)[tok].copy())
    fp["embed"] = errs(D["x"][0], emb)
    for l in range(cfg.n_layer):
        p = f"L{l}."
        x = np.ascontiguousarray(D["x"][l])
        # ---- RMSNorm -> Q8_0 -> QKV GEMV (+ RoPE, K/V rows)
        xq = D["xq_qkv"][l]
        exact[p + "xq_qkv"] = _mismatch(xq, O.quantize_q8_0(O.rms_norm_mul(x, W["attn_norm"][l], cfg.rms_eps)))
        wqkv = np.concatenate([_rows(W["wq"][l], qd), _rows(W["wk"][l], kvd), _rows(W["wv"][l], kvd)])
        if "dots_qkv" in D:
            exact[p + "dots_qkv"] = _mismatch(D["dots_qkv"][l], O.block_dots_q4_0_xq(wqkv, xq))
        qkv = O.mul_mat_q4_0_xq(wqkv, xq)
        q = O.rope_norm(qkv[:qd], hq, Dh, pos, cfg.rope_theta)
        k = O.rope_norm(qkv[qd:qd + kvd], hkv, Dh, pos, cfg.rope_theta)
        v = qkv[qd + kvd:]
        fp[p + "q"] = errs(D["q"][l], q)
        fp[p + "k_row"] = errs(D["k_row"][l].astype(np.float32), k)
        fp[p + "v_row"] = errs(D["v_row"][l].astype(np.float32), v)
        # ---- attention over the cache holding the GPU's own rows at pos
        kc[l][pos] = D["k_row"][l]
        vc[l][pos] = D["v_row"][l]
        att = O.flash_attn_decode(D["q"][l].reshape(hq, Dh), kc[l][:pos + 1].reshape(pos + 1, hkv, Dh),
                                  vc[l][:pos + 1].reshape(pos + 1, hkv, Dh), None).reshape(-1)
        fp[p + "attn"] = errs(D["att"][l], att)
        # ---- O projection from the image the GEMV read
        xq = D["xq_o"][l]
        exact[p + "xq_o"] = _mismatch(xq, O.quantize_q8_0(D["att"][l]))
        if "dots_o" in D:
            exact[p + "dots_o"] = _mismatch(D["dots_o"][l], O.block_dots_q4_0_xq(W["wo"][l], xq))
        fp[p + "x_mid"] = errs(D["x_mid"][l], x + O.mul_mat_q4_0_xq(W["wo"][l], xq))
        # ---- RMSNorm -> Q8_0 -> gate/up GEMV -> SwiGLU
        xm = np.ascontiguousarray(D["x_mid"][l])
        xq = D["xq_gu"][l]
        exact[p + "xq_gu"] = _mismatch(xq, O.quantize_q8_0(O.rms_norm_mul(xm, W["ffn_norm"][l], cfg.rms_eps)))
        if "dots_gu" in D:
            exact[p + "dots_gate"] = _mismatch(D["dots_gu"][l][0::2], O.block_dots_q4_0_xq(W["wgate"][l], xq))
            exact[p + "dots_up"] = _mismatch(D["dots_gu"][l][1::2], O.block_dots_q4_0_xq(W["wup"][l], xq))
        g = O.mul_mat_q4_0_xq(W["wgate"][l], xq)
        u = O.mul_mat_q4_0_xq(W["wup"][l], xq)
        # ggml swiglu in f32: silu(g) = g / (1 + expf(-g)), times u
        h = (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32) * u
        fp[p + "h"] = errs(D["h"][l], h)
        # ---- down projection from the image the SwiGLU epilogue wrote
        xq = D["xq_down"][l]
        exact[p + "xq_down"] = _mismatch(xq, O.quantize_q8_0(D["h"][l]))
        if "dots_down" in D:
            exact[p + "dots_down"] = _mismatch(D["dots_down"][l], O.block_dots_q4_0_xq(W["wdown"][l], xq))
        fp[p + "x_out"] = errs(D["x"][l + 1], xm + O.mul_mat_q4_0_xq(W["wdown"][l], xq))
    # ---- output norm -> Q8_0 -> lm_head
    xf = np.ascontiguousarray(D["x"][cfg.n_layer])
    xq = D["xq_head"]
    exact["xq_head"] = _mismatch(xq, O.quantize_q8_0(O.rms_norm_mul(xf, W["out_norm"], cfg.rms_eps)))
    if "dots_head" in D:
        exact["dots_head"] = _mismatch(D["dots_head"], O.block_dots_q4_0_xq(W["lm_head"], xq))
    fp["logits"] = errs(D["logits"], O.mul_mat_q4_0_xq(W["lm_head"], xq))
    return exact, fp


def assert_stages(exact, fp, tol, what):
    bad = {k: v for k, v in exact.items() if v != 0}
    assert not bad, f"{what}: not bit-exact (mismatching entries): {bad}"
    for k, (nw, ew) in fp.items():
        assert nw <= tol and ew <= tol, f"{what} {k}: normwise {nw:.3e} elementwise {ew:.3e} (tol {tol})"
