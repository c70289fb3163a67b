"""Regenerates the committed golden fixtures in this directory.

Run in the development container (it needs gguf-py and the read-only
reference checkout; neither exists on the GPU box):

    python tests/golden/make_golden.py --reference <path to the reference checkout>

Fixtures written:
  gguf_q8_0.npz / gguf_q4_0.npz
      ggml block bytes and dequantised values produced by gguf-py 0.19.0
      (gguf/quants.py Q8_0 at 378-401, Q4_0 at 220-252; gguf-py states its Q8_0
      is bit-exact with ggml-quants.c).  Inputs: seeded N(0,1), N(0, 0.02^2)
      and hand-made edge blocks (zeros, rounding ties, sign of the max,
      repeated maxima, tiny scales).
  w4a16_probe_golden.npz
      Output of the reference's own W4A16 probe generator
      (experiments/w4a16-gemv/source/gen_data.py), run unmodified in a scratch
      directory: the f16 golden vector and SHA-256 digests of the packed
      weight, scale and broadcast-x files it writes.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def edge_blocks_q8_0() -> np.ndarray:
    b = []
    b.append(np.zeros(32, np.float32))
    # amax 127 -> d = 1, id = 1: exact half-way products test round-half-away
    t = np.array([127.0, 2.5, -2.5, 0.5, -0.5, 1.5, -1.5, 126.5, -126.5, 3.5, -3.5, 0.49999997] + [0.0] * 20,
                 np.float32)
    b.append(t)
    b.append(np.full(32, -3.0, np.float32))
    b.append(np.linspace(-1e-6, 1e-6, 32).astype(np.float32))  # f16 scale underflows
    b.append(np.linspace(-60000.0, 65000.0, 32).astype(np.float32))
    r = np.random.default_rng(7)
    tie = (r.integers(-127, 128, 32).astype(np.float32) + 0.5) * 0.25
    tie[0] = 127.0 * 0.25
    b.append(tie.astype(np.float32))
    return np.stack(b)


def edge_blocks_q4_0() -> np.ndarray:
    b = []
    b.append(np.zeros(32, np.float32))
    t = np.linspace(-1.0, 1.0, 32).astype(np.float32)  # max magnitude at both ends: first wins
    b.append(t)
    t = np.linspace(-2.0, 1.0, 32).astype(np.float32)  # negative max
    b.append(t)
    t = np.full(32, 0.75, np.float32)
    b.append(t)
    t = (np.arange(32, dtype=np.float32) - 16.0) / 2.0  # x*id lands on .5 boundaries
    b.append(t)
    b.append(np.linspace(-1e-6, 2e-6, 32).astype(np.float32))
    return np.stack(b)


def make_quant_fixtures() -> None:
    import gguf  # noqa: F401  (gguf-py 0.19.0)
    from gguf import quants
    from gguf.constants import GGMLQuantizationType as T

    rng = np.random.default_rng(20261201)
    for name, qt, edges in (("q8_0", T.Q8_0, edge_blocks_q8_0()), ("q4_0", T.Q4_0, edge_blocks_q4_0())):
        x_unit = rng.standard_normal((64, 32)).astype(np.float32)
        x_w = (rng.standard_normal((64, 32)) * 0.02).astype(np.float32)
        x = np.concatenate([edges, x_unit, x_w]).reshape(-1)
        blocks = quants.quantize(x.reshape(1, -1), qt)
        deq = quants.dequantize(blocks, qt).reshape(-1).astype(np.float32)
        np.savez_compressed(
            os.path.join(HERE, f"gguf_{name}.npz"),
            x=x,
            blocks=np.asarray(blocks, dtype=np.uint8).reshape(-1),
            dequant=deq,
            n_edge_blocks=np.int32(edges.shape[0]),
        )
        print(f"gguf_{name}.npz: {x.size // 32} blocks")


def sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def make_w4a16_fixture(reference: str) -> None:
    src = os.path.join(reference, "experiments", "w4a16-gemv", "source", "gen_data.py")
    with tempfile.TemporaryDirectory(prefix="w4a16_gen_") as work:
        _make_w4a16_fixture_in(src, work)


def _make_w4a16_fixture_in(src: str, work: str) -> None:
    subprocess.run([sys.executable, src], cwd=work, check=True)
    golden = np.fromfile(os.path.join(work, "output", "golden.bin"), dtype=np.float16)
    np.savez_compressed(
        os.path.join(HERE, "w4a16_probe_golden.npz"),
        golden=golden,
        sha_weight=np.array(sha256(os.path.join(work, "input", "input_weight.bin"))),
        sha_scales=np.array(sha256(os.path.join(work, "input", "input_scales.bin"))),
        sha_x=np.array(sha256(os.path.join(work, "input", "input_x.bin"))),
    )
    print(f"w4a16_probe_golden.npz: golden {golden.shape}")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the read-only reference checkout")
    a = ap.parse_args()
    make_quant_fixtures()
    make_w4a16_fixture(a.reference)


if __name__ == "__main__":
    main()
