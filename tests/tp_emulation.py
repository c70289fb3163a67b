"""Tensor-parallel decode step restated on the CPU (test helper).

Mirrors the sharding of the native model driver (csrc/model.cpp, gen_weight
and enqueue_step) with oracle building blocks and torch.distributed
collectives, so world-size-2 ``gloo`` ranks can check the decomposition
without a GPU:
  * Q/K/V, gate/up and lm_head split by output rows (whole heads for Q/K/V);
  * O and down split by input columns on 32-element block boundaries; rank 0
    adds the residual before the sum (EPI_ADD), the others store (EPI_STORE);
    the partials are summed with an all-reduce;
  * greedy argmax: each rank packs (logit, global row) into an ordered 64-bit
    key (high word: float bits made monotone; low word: ~row, so ties go to
    the lower row) and the ranks take the maximum.
"""
import ctypes as C

import numpy as np

import oracle as O

Q4_BYTES = 18


def rms_norm(x, w, eps):
    y = np.empty_like(x)
    O.lib().ref_rms_norm_mul(O._p(np.ascontiguousarray(x)), O._p(w), O._p(y), x.size, C.c_float(eps))
    return y


def rope(v, n_heads, head_dim, pos, theta):
    v = np.ascontiguousarray(v, dtype=np.float32).copy()
    O.lib().ref_rope_norm(O._p(v), n_heads, head_dim, pos, C.c_float(theta))
    return v


def col_shard(w_blocks, rows, k, c0, nc):
    """Columns [c0, c0+nc) of a Q4_0 matrix [rows][k] (block aligned)."""
    w = w_blocks.reshape(rows, k // 32 * Q4_BYTES)
    return np.ascontiguousarray(w[:, c0 // 32 * Q4_BYTES:(c0 + nc) // 32 * Q4_BYTES])


def row_shard(w_blocks, k, r0, nr):
    w = w_blocks.reshape(-1, k // 32 * Q4_BYTES)
    return np.ascontiguousarray(w[r0:r0 + nr])


def argmax_key(v, row):
    bits = int(np.float32(v).view(np.uint32))
    ordered = (bits ^ 0xFFFFFFFF) if bits & 0x80000000 else (bits | 0x80000000)
    return (ordered << 32) | (0xFFFFFFFF - row)


def key_row(key):
    return 0xFFFFFFFF - (key & 0xFFFFFFFF)


class TpRank:
    """One rank's shard geometry and step, over full host weights."""

    def __init__(self, cfg, W, rank, world):
        self.cfg, self.W, self.rank, self.world = cfg, W, rank, world
        D = cfg["head_dim"]
        self.hq = cfg["n_head"] // world
        self.hkv = cfg["n_head_kv"] // world
        self.ff = cfg["d_ff"] // world
        self.voc = cfg["vocab"] // world
        self.qd, self.kvd = self.hq * D, self.hkv * D

    def attention(self, l, x, pos, kc, vc):
        """Roped q shard and attention output shard; writes this rank's K/V row."""
        c, W, r = self.cfg, self.W, self.rank
        d, D = c["d_model"], c["head_dim"]
        xn = rms_norm(x, W["attn_norm"][l], c["rms_eps"])
        q = O.mul_mat_q4_0(row_shard(W["wq"][l], d, r * self.qd, self.qd), xn)
        k = O.mul_mat_q4_0(row_shard(W["wk"][l], d, r * self.kvd, self.kvd), xn)
        v = O.mul_mat_q4_0(row_shard(W["wv"][l], d, r * self.kvd, self.kvd), xn)
        q = rope(q, self.hq, D, pos, c["rope_theta"])
        k = rope(k, self.hkv, D, pos, c["rope_theta"])
        kc[pos] = k.astype(np.float16)
        vc[pos] = v.astype(np.float16)
        att = O.flash_attn_decode(q.reshape(self.hq, D), kc[:pos + 1].reshape(pos + 1, self.hkv, D),
                                  vc[:pos + 1].reshape(pos + 1, self.hkv, D), None).reshape(-1)
        return q, att

    def o_partial(self, l, x, att):
        c, r = self.cfg, self.rank
        d, hd = c["d_model"], c["n_head"] * c["head_dim"]
        y = O.mul_mat_q4_0(col_shard(self.W["wo"][l], d, hd, r * self.qd, self.qd), att)
        return (y + x).astype(np.float32) if r == 0 else y

    def ffn_partial(self, l, x1):
        c, W, r = self.cfg, self.W, self.rank
        d = c["d_model"]
        xn = rms_norm(x1, W["ffn_norm"][l], c["rms_eps"])
        g = O.mul_mat_q4_0(row_shard(W["wgate"][l], d, r * self.ff, self.ff), xn)
        u = O.mul_mat_q4_0(row_shard(W["wup"][l], d, r * self.ff, self.ff), xn)
        h = ((g / (1.0 + np.exp(-g.astype(np.float64)))) * u).astype(np.float32)
        y = O.mul_mat_q4_0(col_shard(W["wdown"][l], d, c["d_ff"], r * self.ff, self.ff), h)
        return (y + x1).astype(np.float32) if r == 0 else y

    def head(self, x):
        c, W, r = self.cfg, self.W, self.rank
        xn = rms_norm(x, W["out_norm"], c["rms_eps"])
        logits = O.mul_mat_q4_0(row_shard(W["lm_head"], c["d_model"], r * self.voc, self.voc), xn)
        i = int(np.argmax(logits))
        return logits, argmax_key(logits[i], r * self.voc + i)
