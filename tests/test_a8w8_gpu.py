"""The reference add-on's own A8W8 scheme on the GPU (rows a3/a4 of the hot
path): the F16 -> int8 weight transform (per output column s = amax/127 as
f16, q = clamp(round(w/s))) and the one-launch GEMV (x -> f16 -> per-token
int8, exact int32 dot, y = f16(acc * s_x * s_w)).  Bit-exact against the CPU
oracle's restatement of the reference chain (transform patch:1674-1695,
quantize w8a8_quantize_custom_vector.cpp:35-64, matmul
matmul_w8a8_i32_custom.cpp:15-48, dequant at the call site patch:1269-1270),
including the reference's own known answer (custom_a8w8_chain_probe.cpp:189)."""
import numpy as np
import pytest

import oracle as O
import probe_data as PD
from helpers import rng

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def B():
    import b200_decode

    return b200_decode


def unpack(data: np.ndarray, n: int, k: int):
    """Packed A8W8 bytes -> (q int8 [n][k], scales f16 [n])."""
    U = k // 32
    rows = data[: n * 32 * U].view(np.int8).reshape(n, 2, U, 16)
    q = np.concatenate([rows[:, 0], rows[:, 1]], axis=2).reshape(n, k)
    s = data[n * 32 * U: n * 32 * U + 2 * n].view(np.float16)
    return q, s


def oracle_gemv(x: np.ndarray, q_nz: np.ndarray, s: np.ndarray, n: int, k: int):
    xq, xs = O.a8w8_quantize_token(x.astype(np.float16))
    acc = O.a8w8_matmul_i32(xq, q_nz, k, n)
    return O.a8w8_dequant(acc, xs, s).astype(np.float32)


@pytest.mark.parametrize("n,k", [(96, 1536), (64, 512), (160, 8960)])
def test_transform_bit_exact(n, k):
    r = rng(n + k)
    w = (r.standard_normal((n, k)) * 0.02).astype(np.float16)
    w[3] = 0  # an all-zero row takes the 1e-8 floor
    pw = B().a8w8_transform(torch.from_numpy(w).cuda(), n, k)
    q, s = unpack(pw.data.cpu().numpy(), n, k)
    q_nz, s_ref = O.a8w8_transform_weight(w)
    kk = np.arange(k)[None, :]
    nn = np.arange(n)[:, None]
    np.testing.assert_array_equal(q, q_nz[O.a8w8_nz_index(kk, nn, k)])
    np.testing.assert_array_equal(s.view(np.uint16), s_ref.view(np.uint16))


@pytest.mark.parametrize("n,k", [(151936, 1536), (1536, 8960), (8960, 1536), (64, 512), (96, 2048)])
def test_gemv_bit_exact(n, k):
    r = rng(n * 7 + k)
    w = (r.standard_normal((n, k)) * 0.02).astype(np.float16)
    x = (r.standard_normal(k) * 2).astype(np.float32)
    pw = B().a8w8_transform(torch.from_numpy(w).cuda(), n, k)
    y = B().mul_mat(pw, torch.from_numpy(x).cuda()).cpu().numpy()
    q_nz, s = O.a8w8_transform_weight(w)
    np.testing.assert_array_equal(y, oracle_gemv(x, q_nz, s, n, k))
    assert B().device_status(reset=True) == 0


@pytest.mark.parametrize("k,n", [(1536, 8960), (8960, 1536)])
def test_reference_known_answer(k, n):
    """custom_a8w8_chain_probe.cpp: x = 1, w[k][n] = (k % 7) - 3 + (n % 3),
    unit weight scales; out[0] within 8 of sum_k w[k][0]."""
    x16, w, w_nz, expected_first = PD.a8w8_chain_inputs(k, n)
    U = k // 32
    q = w.T.astype(np.int8).reshape(n, U, 32)  # row n = output column n
    packed = np.concatenate([q[:, :, :16].reshape(n, -1), q[:, :, 16:].reshape(n, -1)], axis=1).reshape(-1)
    scales = np.ones(n, np.float16).view(np.uint8)
    pad = (-(2 * n)) % 16
    data = np.concatenate([packed.view(np.uint8), scales, np.zeros(pad, np.uint8)])
    pw = B().PackedWeight(B().TYPE_A8W8, n, k, torch.from_numpy(data).cuda())
    y = B().mul_mat(pw, torch.from_numpy(x16.astype(np.float32)).cuda()).cpu().numpy()
    np.testing.assert_array_equal(y, oracle_gemv(x16.astype(np.float32), w_nz, np.ones(n, np.float16), n, k))
    assert abs(float(y[0]) - expected_first) <= 8.0
