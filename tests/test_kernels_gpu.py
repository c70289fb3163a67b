"""GPU parity of the sm_100a kernels against the CPU oracle, through the C ABI.

Bit-exact: Q8_0 activation bytes and scales, per-block int32 dots, repacked
layouts.  Floating point: max relative error 1e-3 (helpers.TOL).  Shapes are
the four single-kernel benchmark configs (F16 8960 x 1536, GQA 12/2 x 128
over 4096, Q4_0 1536 x 8960, Q8_0 151936 x 1536) plus ragged and boundary
cases the reference's own
probes sweep (attention lengths 1, 127-129, 239-241, 255-257, 511-513, 4096,
8192; GQA ratios 8/2, 16/4, 32/8 as in patch:408-431, 450).
"""
import os

import numpy as np
import pytest

import oracle as O
import probe_data as PD
from helpers import TOL, assert_close, errs, rng

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def B():
    import b200_decode

    return b200_decode


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    assert B().device_status(reset=True) == 0


# ----------------------------------------------------------- activation quant

def test_quantize_q8_0_bit_exact_vs_gguf_fixture():
    f = np.load(os.path.join(GOLD, "gguf_q8_0.npz"))
    x = f["x"].astype(np.float32)
    want = f["blocks"].reshape(-1, 34)
    got = B().quantize_q8_0(dev(x)).cpu().numpy().reshape(-1, 34)
    bad = np.nonzero((got != want).any(axis=1))[0]
    detail = [(int(b), got[b].tolist(), want[b].tolist()) for b in bad[:3]]
    assert bad.size == 0, f"blocks differ: {bad.tolist()} first: {detail}"
    # the same bytes from inside the fused GEMV (its activation export)
    k = x.size
    bw = B()
    pw = bw.repack(bw.TYPE_Q8_0, dev(O.quantize_q8_0(np.ones((3, k), np.float32))), 3, k)
    _, xq = bw.block_dots(pw, dev(x), with_activation=True)
    np.testing.assert_array_equal(xq.cpu().numpy().reshape(-1, 34), want)


@pytest.mark.parametrize("k,scale", [(1536, 1.0), (8960, 1.0), (28672, 30.0), (8192, 1e-4)])
def test_quantize_q8_0_bit_exact_vs_oracle(k, scale):
    x = (rng(k).standard_normal(k) * scale).astype(np.float32)
    got = B().quantize_q8_0(dev(x)).cpu().numpy()
    np.testing.assert_array_equal(got, O.quantize_q8_0(x))


# ---------------------------------------------------------------------- F16

@pytest.mark.parametrize("n,k", [(8960, 1536), (1000, 520), (1, 8), (3, 4096), (33, 16384), (4097, 1024)])
def test_gemv_f16(n, k):
    r = rng(n * 7 + k)
    w = (r.standard_normal((n, k)) * 0.02).astype(np.float16)
    x = r.standard_normal(k).astype(np.float32)
    bw = B()
    pw = bw.repack(bw.TYPE_F16, dev(w), n, k)
    y = bw.mul_mat(pw, dev(x)).cpu().numpy()
    assert_close(y, O.mul_mat_f16(w, x), what=f"f16 {n}x{k}")


@pytest.mark.parametrize("m,n,k", [(2, 8960, 1536), (8, 8960, 1536), (3, 1537, 72), (5, 100, 4096), (8, 16, 8),
                                   (4, 4097, 28672), (7, 1000, 520), (6, 8192, 8192)])
def test_mul_mat_f16_small_m(m, n, k):
    """M <= 8 columns on the F16 weight (tensor cores): every column within the
    bar against the oracle's F16 dot (x rounded to f16, fp32 accumulation).
    Covers ragged rows and k, k past the one-pass shared-memory limit (the
    weight streamed once per column group) and tiny shapes."""
    r = rng(n * 13 + k + m)
    w = (r.standard_normal((n, k)) * 0.02).astype(np.float16)
    x = r.standard_normal((m, k)).astype(np.float32)
    bw = B()
    pw = bw.repack(bw.TYPE_F16, dev(w), n, k)
    y = bw.mul_mat(pw, dev(x)).cpu().numpy()
    assert y.shape == (m, n)
    for j in range(m):
        assert_close(y[j], O.mul_mat_f16(w, x[j]), what=f"f16 small-M {m}x{n}x{k} column {j}")
    assert bw.device_status() == 0


@pytest.mark.parametrize("pad", [24, 3])
def test_mul_mat_f16_small_m_strided(pad):
    """Row strides of x and y larger than k and n (ggml views; pad 3 leaves x
    rows unaligned to 16 bytes); columns of y past n are not written."""
    torch = pytest.importorskip("torch")
    m, n, k = 5, 3000, 1024
    r = rng(5 + pad)
    w = (r.standard_normal((n, k)) * 0.02).astype(np.float16)
    xf = r.standard_normal((m, k + pad)).astype(np.float32)
    bw = B()
    pw = bw.repack(bw.TYPE_F16, dev(w), n, k)
    xd = dev(xf)[:, :k]
    yd = torch.full((m, n + 40), 7.0, dtype=torch.float32, device="cuda")
    bw.mul_mat(pw, xd, y=yd[:, :n])
    y = yd.cpu().numpy()
    for j in range(m):
        assert_close(y[j, :n], O.mul_mat_f16(w, xf[j, :k]), what=f"strided column {j}")
    assert (y[:, n:] == 7.0).all()


def test_gemv_f16_linearity_full_size():
    """Size-independent property at config 1: y(x1 + x2) = y(x1) + y(x2)
    up to f16 rounding of the activation."""
    n, k = 8960, 1536
    r = rng(99)
    w = (r.standard_normal((n, k)) * 0.02).astype(np.float16)
    x1 = r.standard_normal(k).astype(np.float16).astype(np.float32)
    x2 = (r.standard_normal(k) * 2).astype(np.float16).astype(np.float32)
    bw = B()
    pw = bw.repack(bw.TYPE_F16, dev(w), n, k)
    xs = (x1 + x2).astype(np.float16).astype(np.float32)
    y1, y2, y12 = (bw.mul_mat(pw, dev(v)).cpu().numpy() for v in (x1, x2, xs))
    a, _ = errs(y12, O.mul_mat_f16(w, xs))
    assert a <= TOL
    assert errs(y1 + y2, y12)[0] <= 5e-3


# --------------------------------------------------------------------- Q4_0

def q4_inputs(n, k, seed):
    r = rng(seed)
    wf = (r.standard_normal((n, k)) * 0.02).astype(np.float32)
    blocks = O.quantize_q4_0(wf)
    x = r.standard_normal(k).astype(np.float32)
    return blocks, x


@pytest.mark.parametrize("n,k", [(1536, 8960), (10240, 8192), (8192, 28672), (77, 96), (1, 32), (31, 2048)])
def test_gemv_q4_0_ggml_mode(n, k):
    blocks, x = q4_inputs(n, k, n + k)
    bw = B()
    pw = bw.repack(bw.TYPE_Q4_0, dev(blocks), n, k)
    y = bw.mul_mat(pw, dev(x)).cpu().numpy()
    assert_close(y, O.mul_mat_q4_0(blocks, x, mode=0), what=f"q4_0 {n}x{k}")


@pytest.mark.parametrize("n,k", [(1536, 8960), (300, 8960), (65, 64)])
def test_gemv_q4_0_block_dots_bit_exact(n, k):
    blocks, x = q4_inputs(n, k, 3 * n + k)
    bw = B()
    pw = bw.repack(bw.TYPE_Q4_0, dev(blocks), n, k)
    dots, xq = bw.block_dots(pw, dev(x), with_activation=True)
    np.testing.assert_array_equal(dots.cpu().numpy(), O.block_dots("q4_0", blocks, x))
    np.testing.assert_array_equal(xq.cpu().numpy(), O.quantize_q8_0(x))


@pytest.mark.parametrize("n,k", [(1536, 8960), (8960, 1536), (100, 64)])
def test_gemv_q4_0_w4a16_mode(n, k):
    blocks, x = q4_inputs(n, k, 5 * n + k)
    bw = B()
    pw = bw.repack(bw.TYPE_Q4_0, dev(blocks), n, k)
    y = bw.mul_mat(pw, dev(x), q4_mode=bw.Q4_MODE_W4A16).cpu().numpy()
    assert_close(y, O.mul_mat_q4_0(blocks, x, mode=1), what=f"w4a16 {n}x{k}")
    # the two modes differ by the Q8_0 rounding of x only
    y0 = bw.mul_mat(pw, dev(x)).cpu().numpy()
    assert errs(y0, y)[0] < 2e-2


def test_gemv_w4a16_reference_probe_golden():
    """The reference W4A16 probe's weights and x (gen_data.py, seed 20260916)
    as Q4_0 blocks; the GPU W4A16 GEMV meets the reference verifier's
    rtol = atol = 2e-2 against the probe's f16 golden (verify_result.py:15)."""
    f = np.load(os.path.join(GOLD, "w4a16_probe_golden.npz"))
    x16, q, scales = PD.w4a16_probe_inputs()
    blocks = PD.w4a16_as_q4_0_blocks(q, scales)
    bw = B()
    pw = bw.repack(bw.TYPE_Q4_0, dev(blocks), PD.W4_N, PD.W4_K)
    y = bw.mul_mat(pw, dev(x16.astype(np.float32)), q4_mode=bw.Q4_MODE_W4A16).cpu().numpy()
    g = f["golden"].astype(np.float32)
    assert np.allclose(y, g, rtol=2e-2, atol=2e-2)
    assert_close(y, O.mul_mat_q4_0(blocks, x16.astype(np.float32), mode=1), what="probe w4a16")


# --------------------------------------------------------------------- Q8_0

@pytest.mark.parametrize("n,k", [(151936, 1536), (1536, 8960), (5, 32), (257, 4096)])
def test_gemv_q8_0_q8_0(n, k):
    r = rng(n + 2 * k)
    blocks = O.quantize_q8_0((r.standard_normal((n, k)) * 0.02).astype(np.float32))
    x = r.standard_normal(k).astype(np.float32)
    bw = B()
    pw = bw.repack(bw.TYPE_Q8_0, dev(blocks), n, k)
    y = bw.mul_mat(pw, dev(x)).cpu().numpy()
    assert_close(y, O.mul_mat_q8_0(blocks, x), what=f"q8_0 {n}x{k}")


def test_gemv_q8_0_block_dots_bit_exact_full_size():
    n, k = 151936, 1536
    r = rng(4)
    blocks = O.quantize_q8_0((r.standard_normal((n, k)) * 0.02).astype(np.float32))
    x = r.standard_normal(k).astype(np.float32)
    bw = B()
    pw = bw.repack(bw.TYPE_Q8_0, dev(blocks), n, k)
    dots, xq = bw.block_dots(pw, dev(x), with_activation=True)
    np.testing.assert_array_equal(dots.cpu().numpy(), O.block_dots("q8_0", blocks, x))
    np.testing.assert_array_equal(xq.cpu().numpy(), O.quantize_q8_0(x))


def test_repack_interleave2_matches_separate():
    n, k = 96, 2048
    r = rng(8)
    a = O.quantize_q4_0((r.standard_normal((n, k)) * 0.02).astype(np.float32))
    b = O.quantize_q4_0((r.standard_normal((n, k)) * 0.02).astype(np.float32))
    x = r.standard_normal(k).astype(np.float32)
    bw = B()
    pi = bw.repack_interleave2(bw.TYPE_Q4_0, dev(a), dev(b), n, k)
    yi = bw.mul_mat(pi, dev(x)).cpu().numpy()
    ya = bw.mul_mat(bw.repack(bw.TYPE_Q4_0, dev(a), n, k), dev(x)).cpu().numpy()
    yb = bw.mul_mat(bw.repack(bw.TYPE_Q4_0, dev(b), n, k), dev(x)).cpu().numpy()
    np.testing.assert_array_equal(yi[0::2], ya)
    np.testing.assert_array_equal(yi[1::2], yb)


def test_gemv_deterministic():
    n, k = 8960, 1536
    r = rng(12)
    w = (r.standard_normal((n, k)) * 0.02).astype(np.float16)
    x = dev(r.standard_normal(k).astype(np.float32))
    bw = B()
    pw = bw.repack(bw.TYPE_F16, dev(w), n, k)
    ys = [bw.mul_mat(pw, x).cpu().numpy() for _ in range(3)]
    np.testing.assert_array_equal(ys[0], ys[1])
    np.testing.assert_array_equal(ys[0], ys[2])


# ---------------------------------------------------------------- attention

def fa_case(hq, hkv, d, n_kv, seed, tail=0):
    r = rng(seed)
    q = r.standard_normal((hq, d)).astype(np.float32)
    k = r.standard_normal((n_kv, hkv, d)).astype(np.float16)
    v = r.standard_normal((n_kv, hkv, d)).astype(np.float16)
    mask = np.zeros(n_kv, np.float16)
    if tail:
        mask[n_kv - tail:] = -np.inf
    return q, k, v, mask


def run_fa(q, k, v, mask, kv_len=None, scale=None):
    bw = B()
    d = q.shape[1]
    scale = 1.0 / np.sqrt(d) if scale is None else scale
    kl = None if kv_len is None else dev(np.array([kv_len], np.int32))
    out = bw.flash_attn_ext(dev(q), dev(k), dev(v), None if mask is None else dev(mask), scale=scale,
                            kv_lengths=kl)
    return out.cpu().numpy()


def test_fa_config2():
    q, k, v, mask = fa_case(12, 2, 128, 4096, 1)
    out = run_fa(q, k, v, mask)
    assert_close(out, O.flash_attn_decode(q, k, v, mask, mode=0), what="fa config2")


def test_fa_config2_padded_tail_and_kv_len():
    q, k, v, mask = fa_case(12, 2, 128, 4096, 2, tail=1000)
    ref = O.flash_attn_decode(q, k, v, mask, mode=0)
    assert_close(run_fa(q, k, v, mask), ref, what="masked tail")
    kl = int(O.kv_lengths_from_mask(mask)[0])
    assert kl == 3096
    assert_close(run_fa(q, k, v, mask, kv_len=kl), ref, what="kv_len")
    # kv_len alone (no mask) truncates exactly like the reference kernel
    assert_close(run_fa(q, k, v, None, kv_len=kl), O.flash_attn_decode(q, k, v, None, kv_len=kl), what="kv_len only")


@pytest.mark.parametrize("hq,hkv,n_kv", [(64, 8, 4160), (12, 2, 8192)])
def test_fa_three_group_splits_d128(hq, hkv, n_kv):
    """Head dim 128 with 6 or more 64-position chunks per CTA, where the
    launcher runs three warp groups of two stages (the Llama-3-70B attention
    shape has up to 9 chunks per split); also truncated by kv_len so the
    groups end on different chunks."""
    q, k, v, mask = fa_case(hq, hkv, 128, n_kv, n_kv + hq)
    assert_close(run_fa(q, k, v, mask), O.flash_attn_decode(q, k, v, mask, mode=0), what=f"{hq}/{hkv} n_kv={n_kv}")
    kl = n_kv - 77
    assert_close(run_fa(q, k, v, None, kv_len=kl), O.flash_attn_decode(q, k, v, None, kv_len=kl),
                 what=f"{hq}/{hkv} kv_len={kl}")


@pytest.mark.parametrize("n_kv", [1, 2, 63, 64, 65, 127, 128, 129, 239, 240, 241, 255, 256, 257, 511, 512, 513, 8192])
def test_fa_boundary_lengths(n_kv):
    q, k, v, mask = fa_case(14, 2, 64, n_kv, n_kv)
    assert_close(run_fa(q, k, v, mask), O.flash_attn_decode(q, k, v, mask, mode=0), what=f"n_kv={n_kv}")


@pytest.mark.parametrize("hq,hkv,d", [(8, 2, 128), (16, 4, 128), (32, 8, 128), (64, 8, 128), (24, 2, 64),
                                      (4, 4, 256), (40, 8, 128)])
def test_fa_gqa_ratios(hq, hkv, d):
    q, k, v, mask = fa_case(hq, hkv, d, 777, hq * 31 + d)
    assert_close(run_fa(q, k, v, mask), O.flash_attn_decode(q, k, v, mask, mode=0), what=f"{hq}/{hkv} d={d}")


def test_fa_all_masked_gives_zero():
    q, k, v, mask = fa_case(12, 2, 128, 300, 5)
    mask[:] = -np.inf
    out = run_fa(q, k, v, mask)
    assert np.all(out == 0)


def test_fa_vs_reference_kernel_and_ggml_modes():
    """Against the reference AttentionStepCustom semantics (f16 output) the
    difference is the f16 output rounding; against ggml-cpu's f16-V
    accumulator it is that accumulator's own error (reported, looser)."""
    q, k, v, mask = fa_case(12, 2, 128, 4096, 6)
    out = run_fa(q, k, v, mask)
    assert errs(out, O.flash_attn_decode(q, k, v, mask, mode=2))[0] <= 1e-3
    assert errs(out, O.flash_attn_decode(q, k, v, mask, mode=1))[0] <= 5e-2


def test_fa_deterministic_repeats():
    q, k, v, mask = fa_case(12, 2, 128, 4096, 7)
    a = run_fa(q, k, v, mask)
    for _ in range(3):
        np.testing.assert_array_equal(run_fa(q, k, v, mask), a)


def test_fa_strided_cache_view():
    """K/V as a view into a larger cache (kv_size rows allocated, n_kv used):
    ggml's FA view nb1 = Hkv*D*2, nb2 = D*2 over the cache buffer."""
    hq, hkv, d, kv_size, n_kv = 12, 2, 128, 5000, 3000
    r = rng(21)
    kc = r.standard_normal((kv_size, hkv, d)).astype(np.float16)
    vc = r.standard_normal((kv_size, hkv, d)).astype(np.float16)
    q = r.standard_normal((hq, d)).astype(np.float32)
    bw = B()
    kt, vt = dev(kc), dev(vc)
    out = bw.flash_attn_ext(dev(q), kt[:n_kv], vt[:n_kv], None, scale=1 / np.sqrt(d)).cpu().numpy()
    assert_close(out, O.flash_attn_decode(q, kc[:n_kv], vc[:n_kv], None), what="cache view")
