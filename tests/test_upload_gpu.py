"""Chunked weight upload (b200_upload_*), the counterpart of the reference's
set_tensor tracker: a tensor written in arbitrary pieces, in any order, from
several threads, repeats and overlaps included, must become complete exactly
when every byte has arrived, and its packed copy must equal a one-shot
b200_repack of the same bytes.  Also GET_ROWS from the packed Q4_0 copy
(one copy for a tied embedding / output matrix)."""
import threading

import numpy as np
import pytest

import oracle as O
from helpers import rng

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def B():
    import b200_decode

    return b200_decode


def ggml_bytes(wtype, n, k, seed):
    r = rng(seed)
    x = (r.standard_normal((n, k)) * 0.05).astype(np.float32)
    if wtype == B().TYPE_F16:
        return x.astype(np.float16).view(np.uint8).reshape(-1)
    if wtype == B().TYPE_Q4_0:
        return O.quantize_q4_0(x.reshape(-1))
    return O.quantize_q8_0(x.reshape(-1))


def one_shot(wtype, n, k, data):
    src = torch.from_numpy(data.copy()).cuda()
    if wtype == B().TYPE_F16:
        src = src.view(torch.float16).view(n, k)
    return B().repack(wtype, src, n, k).data.cpu().numpy()


@pytest.mark.parametrize("wtype", ["q4_0", "q8_0", "f16"])
def test_sequential_chunks_equal_one_shot_repack(wtype):
    bw = B()
    t = {"q4_0": bw.TYPE_Q4_0, "q8_0": bw.TYPE_Q8_0, "f16": bw.TYPE_F16}[wtype]
    n, k = 96, 1024
    data = ggml_bytes(t, n, k, 1)
    up = bw.Upload(t, n, k)
    step = 1000
    for off in range(0, data.size, step):
        done = up.write(off, data[off:off + step])
        assert done == (off + step >= data.size)
    np.testing.assert_array_equal(up.w.data.cpu().numpy(), one_shot(t, n, k, data))
    assert up.close() == bw.OK


def test_concurrent_overlapping_chunks_complete_once():
    bw = B()
    t, n, k = bw.TYPE_Q4_0, 300, 512
    data = ggml_bytes(t, n, k, 2)
    r = rng(3)
    cuts = np.sort(r.choice(np.arange(1, data.size), size=60, replace=False))
    pieces = list(zip(np.r_[0, cuts], np.r_[cuts, data.size]))
    # repeats and overlapping pieces must not count twice
    pieces += [(int(a), int(min(b + 37, data.size))) for a, b in pieces[:20]]
    order = r.permutation(len(pieces))
    up = bw.Upload(t, n, k)
    completions = []
    lock = threading.Lock()

    def worker(ids):
        for i in ids:
            a, b = pieces[i]
            done = up.write(int(a), data[a:b])
            with lock:
                completions.append(done)

    threads = [threading.Thread(target=worker, args=(order[j::4],)) for j in range(4)]
    for th in threads:
        th.start()
    for th in threads:
        th.join()
    assert completions.count(True) >= 1
    assert up.complete
    got = up.w.data.cpu().numpy()
    np.testing.assert_array_equal(got, one_shot(t, n, k, data))
    idx = torch.tensor([0, 299, 5, 5], dtype=torch.int32, device="cuda")
    rows = bw.get_rows_q4_0_packed(up.w, idx).cpu().numpy()
    np.testing.assert_array_equal(rows, O.dequantize_q4_0(data).reshape(n, k)[[0, 299, 5, 5]])
    assert up.close() == bw.OK


def test_incomplete_and_out_of_range():
    bw = B()
    t, n, k = bw.TYPE_Q4_0, 8, 256
    data = ggml_bytes(t, n, k, 4)
    up = bw.Upload(t, n, k)
    assert not up.write(0, data[:100])
    assert not up.write(0, data[:100])  # the same bytes again: still incomplete
    with pytest.raises(bw.B200Error):
        up.write(data.size - 10, data[:20])  # past the end
    assert up.close() == -6  # B200_ESTATE: never complete
    assert bw.device_status(reset=True) == 0
