"""Restated data generators of the reference's kernel probes (test helpers).

``w4a16_probe_inputs`` repeats the numpy call sequence of the reference W4A16
probe generator (experiments/w4a16-gemv/source/gen_data.py:6-32): seed
20260916, x ~ N(0, 0.08) as f16, int4 weights in [-8, 7], per-(column, group)
f16 scales ~ U(0.002, 0.02), then its tile-448 nibble packing.  The committed
fixture stores SHA-256 digests of the reference's own output files so the
restatement is checked byte for byte.

``a8w8_chain_inputs`` is the known-answer case of the reference A8W8 chain
probe (experiments/a8w8/custom_a8w8_chain_probe.cpp:104-115): x = 1.0 f16 and
W[k, n] = (k % 7) - 3 + (n % 3) stored in int8 NZ 16x32 order, w_scale = 1.
"""
import numpy as np

W4_SEED = 20260916
W4_K = 1536
W4_N = 8960
W4_GROUP = 32
W4_TILE = 448


def w4a16_probe_inputs():
    rng = np.random.default_rng(W4_SEED)
    x = rng.normal(0.0, 0.08, W4_K).astype(np.float16)
    q = rng.integers(-8, 8, size=(W4_N, W4_K), dtype=np.int8)
    scales = rng.uniform(0.002, 0.02, size=(W4_N, W4_K // W4_GROUP)).astype(np.float16)
    return x, q, scales


def w4a16_probe_pack(q, scales):
    tiles = W4_N // W4_TILE
    groups = W4_K // W4_GROUP
    half = W4_TILE // 2
    qq = (q.astype(np.int16) + 8).reshape(tiles, W4_TILE, groups, W4_GROUP)
    low = qq[:, :half].transpose(0, 2, 3, 1)   # [tile][group][k][j]
    high = qq[:, half:].transpose(0, 2, 3, 1)
    packed = (low | (high << 4)).astype(np.uint8)
    sl = scales.reshape(tiles, W4_TILE, groups).transpose(0, 2, 1).astype(np.float16)
    return np.ascontiguousarray(packed), np.ascontiguousarray(sl)


def w4a16_as_q4_0_blocks(q, scales):
    """Re-expresses the probe's int4 weights as ggml Q4_0 blocks: d = the
    group scale, nibble = q + 8 (element j low, element j+16 high)."""
    n, k = q.shape
    nb = k // 32
    qq = (q.astype(np.int16) + 8).astype(np.uint8).reshape(n, nb, 2, 16)
    qs = qq[:, :, 0, :] | (qq[:, :, 1, :] << 4)
    d = scales.astype(np.float16).view(np.uint8).reshape(n, nb, 2)
    return np.ascontiguousarray(np.concatenate([d, qs], axis=-1).reshape(n, nb * 18))


def a8w8_chain_inputs(k, n):
    kk = np.arange(k)[:, None]
    nn = np.arange(n)[None, :]
    w = ((kk % 7) - 3 + (nn % 3)).astype(np.int8)      # [k][n]
    idx = ((((nn // 32) * (k // 16) + kk // 16) * 16 + kk % 16) * 32 + nn % 32)
    w_nz = np.empty(k * n, dtype=np.int8)
    w_nz[idx.reshape(-1)] = w.reshape(-1)
    x = np.ones(k, dtype=np.float16)
    expected_first = int(w[:, 0].astype(np.int64).sum())
    return x, w, w_nz, expected_first
