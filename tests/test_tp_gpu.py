"""Tensor-parallel model parity on 2 GPUs (skipped with fewer).

Runs tests/tp_worker.py under torchrun: the native driver with tp_world = 2
(NCCL all-reduces after O and down, vocab-parallel lm_head with a max
all-reduce of packed argmax keys).  Rank 0 reassembles the shards and checks
every stage per layer against the unsharded oracle with the same bars as the
single-GPU model test; the residual stream must be identical on both ranks
and the captured-graph greedy tokens must agree."""
import json
import os
import socket
import subprocess
import sys

import pytest

from helpers import TOL

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("allreduce", ["peer", "fused"])
def test_tp2_model_per_layer_parity(tmp_path, allreduce):
    """peer: the one-shot all-reduce kernel after O and down; fused: the O /
    down epilogue pushes its rows to every rank and the next GEMV's prologue
    sums them (layer-dump steps keep the kernel, so the graph step's logits
    are also compared bit for bit with a layer-dump step's)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    out = tmp_path / "tp2.json"
    cmd = ["timeout", "-k", "60", "900", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "tp_worker.py"), "--out", str(out)]
    env = dict(os.environ)
    env.pop("B200_TP_ALLREDUCE", None)
    if allreduce == "fused":
        env["B200_TP_ALLREDUCE"] = "fused"
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    rep = json.loads(out.read_text())
    assert rep["status"] == 0
    assert rep["x_replicated"]
    assert rep["greedy"][0] == rep["greedy"][1]
    assert all(rep["graph_vs_dump_equal"])
    for i, (ex, st) in enumerate(zip(rep["exact"], rep["stages"])):
        bad = {k: v for k, v in ex.items() if v != 0}
        assert not bad, f"step {i}: not bit-exact: {bad}"
        for k, (nw, ew) in st.items():
            assert nw <= TOL and ew <= TOL, f"step {i} {k}: normwise {nw:.3e} elementwise {ew:.3e}"


@pytest.mark.parametrize("world", [4, 8])
def test_tp_model_per_layer_parity_more_ranks(tmp_path, world):
    """The same per-layer check on 4 and 8 ranks (a model with eight KV
    heads, one to four per rank), peer all-reduce; skipped with fewer GPUs."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = tmp_path / f"tp{world}.json"
    cmd = ["timeout", "-k", "60", "900", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "tp_worker.py"), "--out", str(out), "--shape", "small8"]
    env = dict(os.environ)
    env.pop("B200_TP_ALLREDUCE", None)
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    errs = [ln for ln in r.stderr.splitlines() if "Error" in ln or "error" in ln or "Traceback" in ln]
    assert r.returncode == 0, r.stdout[-2000:] + "\n".join(errs[:40]) + r.stderr[:3000]
    rep = json.loads(out.read_text())
    assert "error" not in rep, rep["error"]
    assert rep["status"] == 0 and rep["world"] == world
    assert rep["x_replicated"]
    assert len(set(map(tuple, rep["greedy"]))) == 1
    assert all(rep["graph_vs_dump_equal"])
    for i, (ex, st) in enumerate(zip(rep["exact"], rep["stages"])):
        bad = {k: v for k, v in ex.items() if v != 0}
        assert not bad, f"step {i}: not bit-exact: {bad}"
        for k, (nw, ew) in st.items():
            assert nw <= TOL and ew <= TOL, f"step {i} {k}: normwise {nw:.3e} elementwise {ew:.3e}"
