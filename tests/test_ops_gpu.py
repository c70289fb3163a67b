"""GPU parity of the standalone neighbour ops (ggml RMS_NORM + MUL, ROPE,
SET_ROWS, GET_ROWS, SWIGLU, ADD, ARGMAX) against the CPU oracle, through the
C ABI.  Bit-exact where the arithmetic is fully specified (RMS_NORM with a
double sum, f16 conversion, Q4_0 dequantisation, add, argmax); within a few
ulp where CUDA's sin/cos/exp stand in for the C library's (ROPE, SWIGLU)."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
from helpers import rng

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def B():
    import b200_decode

    return b200_decode


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert B().device_status(reset=True) == 0


@pytest.mark.parametrize("n,rows", [(8192, 1), (1536, 3), (4096, 2), (100, 1)])
def test_rms_norm_mul_bit_exact(n, rows):
    r = rng(n + rows)
    x = (r.standard_normal((rows, n)) * 3).astype(np.float32)
    w = (1 + 0.1 * r.standard_normal(n)).astype(np.float32)
    got = B().rms_norm(dev(x), 1e-5, w=dev(w)).cpu().numpy()
    for i in range(rows):
        ref = np.empty(n, np.float32)
        O.lib().ref_rms_norm_mul(O._p(x[i]), O._p(w), O._p(ref), n, C.c_float(1e-5))
        np.testing.assert_array_equal(got[i], ref)
    plain = B().rms_norm(dev(x), 1e-5).cpu().numpy()
    ones = np.ones(n, np.float32)
    ref = np.empty(n, np.float32)
    O.lib().ref_rms_norm_mul(O._p(x[0]), O._p(ones), O._p(ref), n, C.c_float(1e-5))
    np.testing.assert_array_equal(plain[0], ref)


@pytest.mark.parametrize("n_heads,head_dim,pos", [(64, 128, 4100), (8, 64, 0), (2, 128, 123456), (12, 128, 1)])
def test_rope_norm_matches_oracle(n_heads, head_dim, pos):
    r = rng(pos + head_dim)
    x = r.standard_normal((2, n_heads, head_dim)).astype(np.float32)
    got = B().rope_norm(dev(x), dev(np.array([pos, pos + 7], np.int32)), 500000.0).cpu().numpy()
    for t, p in enumerate((pos, pos + 7)):
        ref = x[t].copy().reshape(-1)
        O.lib().ref_rope_norm(O._p(ref), n_heads, head_dim, p, C.c_float(500000.0))
        d = np.abs(got[t].reshape(-1) - ref).max() / np.abs(ref).max()
        assert d <= 2e-6, f"rope pos {p}: {d:.3e}"


def test_set_rows_f16_bit_exact_and_bounds():
    r = rng(3)
    kv_size, n = 96, 256
    cache = torch.zeros((kv_size, n + 64), dtype=torch.float16, device="cuda")[:, :n]
    src = r.standard_normal((3, n)).astype(np.float32) * 10
    idx = np.array([5, 95, 40], np.int64)
    B().set_rows_f16(dev(src), dev(idx), cache)
    c = cache.cpu().numpy()
    for i, row in enumerate(idx):
        np.testing.assert_array_equal(c[row].view(np.uint16), src[i].astype(np.float16).view(np.uint16))
    assert np.count_nonzero(c.view(np.uint16)) == np.count_nonzero(src.astype(np.float16).view(np.uint16))


def test_set_rows_out_of_range_reports_bounds():
    cache = torch.zeros((8, 64), dtype=torch.float16, device="cuda")
    B().set_rows_f16(dev(np.ones((1, 64), np.float32)), dev(np.array([8], np.int64)), cache)
    assert B().device_status(reset=True) == 2  # B200_DEVSTATUS_BOUNDS
    assert int(torch.count_nonzero(cache)) == 0


def test_get_rows_q4_0_bit_exact_and_bounds():
    r = rng(4)
    vocab, n = 300, 512
    table = O.quantize_q4_0((r.standard_normal((vocab, n)) * 0.05).astype(np.float32).reshape(-1))
    idx = np.array([0, 299, 17, 17], np.int32)
    got = B().get_rows_q4_0(dev(table), dev(idx), vocab, n).cpu().numpy()
    ref = O.dequantize_q4_0(table).reshape(vocab, n)[idx]
    np.testing.assert_array_equal(got, ref)
    bad = B().get_rows_q4_0(dev(table), dev(np.array([vocab, -1], np.int32)), vocab, n).cpu().numpy()
    assert B().device_status(reset=True) == 2
    assert np.all(bad == 0)


def test_swiglu_add_argmax():
    r = rng(5)
    n = 28672
    g = (r.standard_normal(n) * 4).astype(np.float32)
    u = r.standard_normal(n).astype(np.float32)
    got = B().swiglu(dev(g), dev(u)).cpu().numpy()
    ref = (g.astype(np.float64) / (1 + np.exp(-g.astype(np.float64))) * u).astype(np.float32)
    assert np.abs(got - ref).max() / np.abs(ref).max() <= 2e-6
    a, b = r.standard_normal(n).astype(np.float32), r.standard_normal(n).astype(np.float32)
    np.testing.assert_array_equal(B().add(dev(a), dev(b)).cpu().numpy(), a + b)
    x = r.standard_normal(151936).astype(np.float32)
    assert int(B().argmax(dev(x)).item()) == int(O.lib().ref_argmax(O._p(x), x.size)) == int(np.argmax(x))
    t = np.full(1000, -np.inf, np.float32)
    t[[10, 500, 900]] = 2.5  # ties: the first maximum
    assert int(B().argmax(dev(t)).item()) == 10
    t2 = -np.abs(r.standard_normal(77)).astype(np.float32) - 1.0
    assert int(B().argmax(dev(t2)).item()) == int(np.argmax(t2))
