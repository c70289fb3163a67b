"""The allocation-free attention entry point, b200_fa_decode_static_scratch.

It serves hosts that cannot allocate device memory when attention runs; its
split-KV partials live in a fixed per-device array of the library.  The GPU
test checks it against b200_fa_decode (the workspace entry point) through
the C ABI, on two calls in a row with different shapes, so the second call
runs on the array the first one left behind, and against the CPU oracle
(fp64 attention of the same inputs), so that the head dim 256 case -- where
both entry points run the same CUDA-core kernel -- also meets an
independent answer.  This file is named to be collected last and passes
alone in a fresh process as well as after the other tests.
"""
import ctypes as C

import numpy as np
import pytest

from helpers import TOL, assert_close, rng


def B():
    import b200_decode

    return b200_decode


def test_static_scratch_rejects_oversized_request_without_device():
    """Rejected before any CUDA call: 8192 query heads of dim 256 need more
    partial space than the fixed array holds."""
    bw = B()
    L = bw.lib()
    hq, hkv, d, n_kv = 8192, 1024, 256, 64
    assert L.b200_fa_workspace_size(d, hq, hkv, n_kv) > bw.FA_STATIC_SCRATCH_BYTES
    fake = C.c_void_p(4096)
    rc = L.b200_fa_decode_static_scratch(fake, fake, fake, None, None, fake, d, hq, hkv, n_kv, hkv * d * 2, d * 2,
                                         hkv * d * 2, d * 2, 1.0, None)
    assert rc == bw.ESCRATCH
    assert b"static scratch" in L.b200_strerror(rc)
    # argument errors come first, as in b200_fa_decode
    assert L.b200_fa_decode_static_scratch(None, fake, fake, None, None, fake, 128, 8, 2, 64, 512, 256, 512, 256,
                                           1.0, None) == bw.EINVAL


CASES = {
    "config2": (12, 2, 128, 4096, 1000),  # hq, hkv, head_dim, n_kv, masked tail
    "llama70b": (64, 8, 128, 4160, 0),
    "d64": (24, 2, 64, 513, 17),
    "d256": (4, 4, 256, 777, 0),
}


def _case(name, seed):
    hq, hkv, d, n_kv, tail = CASES[name]
    r = rng(seed)
    q = r.standard_normal((hq, d)).astype(np.float32)
    k = r.standard_normal((n_kv, hkv, d)).astype(np.float16)
    v = r.standard_normal((n_kv, hkv, d)).astype(np.float16)
    mask = np.zeros(n_kv, np.float16)
    if tail:
        mask[n_kv - tail:] = -np.inf
    return q, k, v, mask


def _both(torch, q, k, v, mask, kv_len=None):
    """(static-scratch result, workspace-entry result); both are also held
    to the CPU oracle here."""
    import oracle as O

    bw = B()
    dq, dk, dv, dm = (torch.from_numpy(a).cuda() for a in (q, k, v, mask))
    kl = None if kv_len is None else torch.tensor([kv_len], dtype=torch.int32, device="cuda")
    scale = 1.0 / np.sqrt(q.shape[1])
    ref = bw.flash_attn_ext(dq, dk, dv, dm, scale=scale, kv_lengths=kl).cpu().numpy()
    out = torch.full_like(dq, float("nan"))
    got = bw.flash_attn_ext_static_scratch(dq, dk, dv, dm, scale=scale, kv_lengths=kl, out=out)
    assert got.data_ptr() == out.data_ptr()
    got = got.cpu().numpy()
    truth = O.flash_attn_decode(q, k, v, mask, kv_len=kv_len, scale=scale)
    assert_close(got, truth, tol=TOL, what="static scratch vs oracle")
    assert_close(ref, truth, tol=TOL, what="workspace entry vs oracle")
    return got, ref


@pytest.mark.gpu
@pytest.mark.parametrize("first,second", [("config2", "llama70b"), ("llama70b", "d64"), ("d256", "config2")])
def test_static_scratch_matches_workspace_entry_two_calls_in_a_row(first, second):
    torch = pytest.importorskip("torch")
    bw = B()
    for i, name in enumerate((first, second)):
        q, k, v, mask = _case(name, 100 + i + 7 * len(name))
        got, ref = _both(torch, q, k, v, mask)
        assert np.all(np.isfinite(got)), name
        assert_close(got, ref, tol=TOL, what=f"static scratch {name} (call {i + 1})")
    assert bw.device_status(reset=True) == 0


@pytest.mark.gpu
def test_static_scratch_kv_len_and_oversized_request_on_device():
    """kv_len truncation as in b200_fa_decode; an oversized request returns
    ESCRATCH with nothing launched, and the next call is unaffected."""
    torch = pytest.importorskip("torch")
    bw = B()
    q, k, v, mask = _case("config2", 5)
    got, ref = _both(torch, q, k, v, mask, kv_len=3096)
    assert_close(got, ref, tol=TOL, what="static scratch kv_len")

    hq, hkv, d, n_kv = 8192, 1024, 256, 64
    big_q = torch.zeros((hq, d), dtype=torch.float32, device="cuda")
    big_kv = torch.zeros((n_kv, hkv, d), dtype=torch.float16, device="cuda")
    with pytest.raises(bw.B200Error) as ei:
        bw.flash_attn_ext_static_scratch(big_q, big_kv, big_kv, None, scale=1.0)
    assert ei.value.code == bw.ESCRATCH

    got2, ref2 = _both(torch, q, k, v, mask)
    assert_close(got2, ref2, tol=TOL, what="static scratch after rejection")
    assert bw.device_status(reset=True) == 0
