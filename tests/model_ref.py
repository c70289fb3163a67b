"""Per-layer teacher forcing for whole-model parity (test helper).

Q8_0 activation quantisation is discontinuous: ulp-level differences in fp32
accumulation order between two valid implementations flip single int8 values,
and random-init weights (N(0, 0.02^2), unit norms) let the residual stream
grow, so such flips amplify across layers.  The parity check therefore feeds
the GPU's own layer input (from b200_model_debug_step) to the oracle for every
layer and compares that layer's outputs; the final norm + lm_head are checked
the same way from the GPU's last residual."""
import ctypes as C

import numpy as np

import oracle as O
from helpers import errs


def per_layer_errors(cfg, W, kc, vc, x, q, a, logits, tok, pos):
    """Errors of every stage given the GPU's inputs.  kc/vc (oracle caches) get
    this step's K/V rows written.  Returns {stage: (normwise, elementwise)}."""
    L = O.lib()
    d, D, hq, hkv = cfg.d_model, cfg.head_dim, cfg.n_head, cfg.n_head_kv
    out = {}
    emb = O.dequantize_q4_0(W["tok_embd"].reshape(cfg.vocab, -1)[tok].copy())
    out["embed"] = errs(x[0], emb)
    for l in range(cfg.n_layer):
        xl = np.ascontiguousarray(x[l])
        xn = np.empty(d, np.float32)
        L.ref_rms_norm_mul(O._p(xl), O._p(W["attn_norm"][l]), O._p(xn), d, C.c_float(cfg.rms_eps))
        qq = O.mul_mat_q4_0(W["wq"][l], xn)
        kk = O.mul_mat_q4_0(W["wk"][l], xn)
        vv = O.mul_mat_q4_0(W["wv"][l], xn)
        L.ref_rope_norm(O._p(qq), hq, D, pos, C.c_float(cfg.rope_theta))
        L.ref_rope_norm(O._p(kk), hkv, D, pos, C.c_float(cfg.rope_theta))
        out[f"L{l}.q"] = errs(q[l], qq)
        kc[l][pos] = kk.astype(np.float16)
        vc[l][pos] = vv.astype(np.float16)
        att = O.flash_attn_decode(q[l].reshape(hq, D), kc[l][:pos + 1].reshape(pos + 1, hkv, D),
                                  vc[l][:pos + 1].reshape(pos + 1, hkv, D), None).reshape(-1)
        out[f"L{l}.attn"] = errs(a[l], att)
        y = O.mul_mat_q4_0(W["wo"][l], np.ascontiguousarray(a[l]))
        x1 = (xl + y).astype(np.float32)
        xn2 = np.empty(d, np.float32)
        L.ref_rms_norm_mul(O._p(x1), O._p(W["ffn_norm"][l]), O._p(xn2), d, C.c_float(cfg.rms_eps))
        g = O.mul_mat_q4_0(W["wgate"][l], xn2)
        u = O.mul_mat_q4_0(W["wup"][l], xn2)
        h = ((g / (1.0 + np.exp(-g.astype(np.float64)))) * u).astype(np.float32)
        y2 = O.mul_mat_q4_0(W["wdown"][l], h)
        out[f"L{l}.x_out"] = errs(x[l + 1], x1 + y2)
    xn = np.empty(d, np.float32)
    xf = np.ascontiguousarray(x[cfg.n_layer])
    L.ref_rms_norm_mul(O._p(xf), O._p(W["out_norm"]), O._p(xn), d, C.c_float(cfg.rms_eps))
    out["logits"] = errs(logits, O.mul_mat_q4_0(W["lm_head"], xn))
    return out
