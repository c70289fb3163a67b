"""Tensor-parallel decomposition on CPU: two ``gloo`` ranks against one.

Each rank runs its shard of a decode step (tp_emulation.TpRank, the split
the native driver uses) with all-reduces over gloo.  Every stage is checked
against the unsharded oracle, teacher-forced on the ranks' own stage inputs:
  * roped q and attention outputs are bit-identical to the unsharded ones
    (whole heads per rank, identical Q8_0 blocks);
  * the O and down all-reduces differ from one unsharded sum only in the
    order of a two-term fp32 addition (normwise <= 1e-5);
  * logits shards are bit-identical and the packed-key max picks the global
    argmax, lowest row on ties.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

CFG = dict(n_layer=2, d_model=256, n_head=8, n_head_kv=4, head_dim=64, d_ff=512, vocab=512, kv_size=48,
           rope_theta=10000.0, rms_eps=1e-5)
N_PREFILL = 20


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def model_weights(cfg, seed=5):
    import oracle as O

    d, hd, ff = cfg["d_model"], cfg["n_head"] * cfg["head_dim"], cfg["d_ff"]
    kvd = cfg["n_head_kv"] * cfg["head_dim"]
    L = cfg["n_layer"]
    s = iter(range(seed * 1000, seed * 1000 + 100))
    W = {"tok_embd": O.synth_q4_0(next(s), 0.02, 0, cfg["vocab"], d),
         "lm_head": O.synth_q4_0(next(s), 0.02, 0, cfg["vocab"], d)}
    shapes = {"wq": (hd, d), "wk": (kvd, d), "wv": (kvd, d), "wo": (d, hd), "wgate": (ff, d), "wup": (ff, d),
              "wdown": (d, ff)}
    for key, (rows, k) in shapes.items():
        W[key] = [O.synth_q4_0(next(s), 0.02, 0, rows, k) for _ in range(L)]
    r = np.random.default_rng(seed)
    W["attn_norm"] = [(1 + 0.1 * r.standard_normal(d)).astype(np.float32) for _ in range(L)]
    W["ffn_norm"] = [(1 + 0.1 * r.standard_normal(d)).astype(np.float32) for _ in range(L)]
    W["out_norm"] = (1 + 0.1 * r.standard_normal(d)).astype(np.float32)
    kc = [np.zeros((cfg["kv_size"], kvd), np.float16) for _ in range(L)]
    vc = [np.zeros((cfg["kv_size"], kvd), np.float16) for _ in range(L)]
    for l in range(L):
        kc[l][:N_PREFILL] = r.standard_normal((N_PREFILL, kvd)).astype(np.float16)
        vc[l][:N_PREFILL] = r.standard_normal((N_PREFILL, kvd)).astype(np.float16)
    return W, kc, vc


def _rank_main(rank, world, port, result_dir):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        import oracle as O
        import tp_emulation as T
        from helpers import errs

        cfg = CFG
        W, kc, vc = model_weights(cfg)
        tr = T.TpRank(cfg, W, rank, world)
        # this rank's KV heads: columns [rank*kvd_l, (rank+1)*kvd_l) of the cache
        kc_r = [np.ascontiguousarray(k[:, rank * tr.kvd:(rank + 1) * tr.kvd]) for k in kc]
        vc_r = [np.ascontiguousarray(v[:, rank * tr.kvd:(rank + 1) * tr.kvd]) for v in vc]
        full = T.TpRank(cfg, W, 0, 1)

        def allreduce(a):
            t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
            dist.all_reduce(t)
            return t.numpy()

        def gather(a):
            parts = [torch.zeros(a.size, dtype=torch.float32) for _ in range(world)]
            dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)))
            return np.concatenate([p.numpy() for p in parts])

        report = {}
        tok, pos = 17, N_PREFILL
        x = O.dequantize_q4_0(W["tok_embd"].reshape(cfg["vocab"], -1)[tok].copy())
        kc_f = [k.copy() for k in kc]
        vc_f = [v.copy() for v in vc]
        for l in range(cfg["n_layer"]):
            q, att = tr.attention(l, x, pos, kc_r[l], vc_r[l])
            q_all, att_all = gather(q), gather(att)
            q_ref, att_ref = full.attention(l, x, pos, kc_f[l], vc_f[l])
            report[f"L{l}.q_exact"] = bool(np.array_equal(q_all, q_ref))
            report[f"L{l}.attn_exact"] = bool(np.array_equal(att_all, att_ref))
            x1 = allreduce(tr.o_partial(l, x, att))
            report[f"L{l}.o"] = errs(x1, full.o_partial(l, x, att_all))[0]
            x2 = allreduce(tr.ffn_partial(l, x1))
            report[f"L{l}.ffn"] = errs(x2, full.ffn_partial(l, x1))[0]
            x = x2
        logits, key = tr.head(x)
        logits_all = gather(logits)
        ref_logits, ref_key = full.head(x)
        report["logits_exact"] = bool(np.array_equal(logits_all, ref_logits))
        # ordered u64 key -> i64 (shift by 2^63 keeps the order), max over ranks, back
        kt = torch.tensor([key - (1 << 63)], dtype=torch.int64)
        dist.all_reduce(kt, op=dist.ReduceOp.MAX)
        gkey = int(kt.item()) + (1 << 63)
        report["argmax"] = T.key_row(gkey)
        report["argmax_ref"] = int(np.argmax(ref_logits))
        report["key_ref"] = ref_key == gkey
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), np.array([report], dtype=object))
    finally:
        dist.destroy_process_group()


def test_tp2_gloo_decomposition_matches_unsharded(tmp_path):
    import torch.multiprocessing as mp

    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for rank in range(world):
        rep = np.load(tmp_path / f"rank{rank}.npy", allow_pickle=True)[0]
        for key, val in rep.items():
            if key.endswith("_exact") or key == "key_ref":
                assert val, f"rank {rank}: {key}"
            elif key.endswith(".o") or key.endswith(".ffn"):
                assert val <= 1e-5, f"rank {rank}: {key} = {val:.3e}"
        assert rep["argmax"] == rep["argmax_ref"]


def test_argmax_key_orders_like_argmax():
    import tp_emulation as T

    vals = np.array([-3.0, -0.0, 0.0, 1e-30, 2.5, 2.5, -np.inf, 7.0, 7.0], np.float32)
    keys = [T.argmax_key(v, i) for i, v in enumerate(vals)]
    assert T.key_row(max(keys)) == int(np.argmax(vals)) == 7
    assert T.key_row(max(keys[:6])) == 4  # tie 2.5 at rows 4 and 5 -> lower row
    assert T.argmax_key(-1.0, 0) < T.argmax_key(-0.5, 0) < T.argmax_key(0.25, 0)
