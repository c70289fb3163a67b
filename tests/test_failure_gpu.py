"""Failure detection on one GPU, without faulting it.

* A bounded device-side wait runs out: the one-shot all-reduce kernel is
  launched with world = 2 where the second rank's announcement is a flag in
  local memory that nothing writes.  The kernel must give up after the wait
  limit, record B200_DEVSTATUS_TIMEOUT and return; while the bit is set a
  later collective gives up at once (a dead peer costs one limit per step,
  not one per collective); once the host clears the word and the "peer"
  arrives, the same call completes with the rank-ordered sum.
* Device memory exhaustion is an error code (B200_ENOMEM), not a crash, and
  the device stays usable afterwards.
"""
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _B():
    import b200_decode as B

    return B


def _ar(B, x, a, b, flags, peer, seq):
    B.tp_allreduce_f32(x, [a, b], 0, flags, [flags.data_ptr(), peer.data_ptr()], seq)
    torch.cuda.synchronize()


def test_allreduce_wait_runs_out_is_sticky_and_recovers():
    B = _B()
    B.device_status(reset=True)
    n = 4096
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(n, device="cuda", generator=g)
    b = torch.randn(n, device="cuda", generator=g)
    x = torch.zeros(n, device="cuda")
    flags = torch.zeros(2, dtype=torch.int64, device="cuda")  # this rank's flags: [rank 0, rank 1]
    peer = torch.zeros(2, dtype=torch.int64, device="cuda")   # stands in for rank 1's flag array
    limit_s = 0.2
    try:
        B.set_wait_timeout(int(limit_s * 1e9))
        # rank 1 never announces collective 1: the wait gives up after the limit
        t0 = time.perf_counter()
        _ar(B, x, a, b, flags, peer, 1)
        t1 = time.perf_counter()
        assert t1 - t0 >= 0.9 * limit_s
        assert B.device_status(reset=False) & B.DEVSTATUS_TIMEOUT
        # our own announcements were made (local slot and the peer's slot)
        assert int(flags[0]) == 1 and int(peer[0]) == 1
        # with the timeout recorded, the next collective gives up at once
        t0 = time.perf_counter()
        _ar(B, x, a, b, flags, peer, 2)
        t1 = time.perf_counter()
        assert t1 - t0 < 0.5 * limit_s, f"sticky timeout not honoured: {t1 - t0:.3f} s"
        assert B.device_status(reset=True) & B.DEVSTATUS_TIMEOUT
        # the peer arrives (its announcement of collective 3) and the status is clear: the call completes
        flags[1] = 3
        _ar(B, x, a, b, flags, peer, 3)
        assert B.device_status(reset=True) == 0
        ref = (a.cpu().numpy().astype(np.float32) + b.cpu().numpy().astype(np.float32))
        np.testing.assert_array_equal(x.cpu().numpy(), ref)
    finally:
        B.set_wait_timeout(0)
        B.device_status(reset=True)


def test_allreduce_rejects_bad_arguments():
    B = _B()
    x = torch.zeros(8, device="cuda")
    f = torch.zeros(2, dtype=torch.int64, device="cuda")
    with pytest.raises(B.B200Error):
        B.tp_allreduce_f32(x, [x, x], 2, f, [f.data_ptr(), f.data_ptr()], 1)  # rank out of range
    with pytest.raises(B.B200Error):
        B.tp_allreduce_f32(x, [x, x], 0, f, [f.data_ptr(), f.data_ptr()], 0)  # seq 0
    with pytest.raises(B.B200Error):
        B.tp_allreduce_f32(x[:6], [x, x], 0, f, [f.data_ptr(), f.data_ptr()], 1)  # n not a multiple of 4


def test_model_out_of_device_memory_is_enomem_and_device_stays_usable():
    import decode_model as M

    B = _B()
    # 2^30 cache rows of 2 x 64 halves per layer: 256 GiB per K cache, more than any B200 holds
    cfg = M.LlamaConfig(n_layer=2, d_model=512, n_head=8, n_head_kv=2, head_dim=64, d_ff=1024, vocab=1024,
                        kv_size=1 << 30)
    with pytest.raises(B.B200Error) as ei:
        M.DecodeModel(cfg)
    assert ei.value.code == -4  # B200_ENOMEM
    ok = M.DecodeModel(M.LlamaConfig(n_layer=2, d_model=512, n_head=8, n_head_kv=2, head_dim=64, d_ff=1024,
                                     vocab=1024, kv_size=64))
    ok.init_synthetic(seed=1)
    ok.fill_kv_synthetic(seed=2, n_pos=8)
    t = ok.decode(3, 8)
    assert 0 <= t < 1024
    ok.close()
    assert B.device_status(reset=True) == 0


@pytest.mark.parametrize("fault,code", [("nccl_init", -5), ("alloc:1", -4), ("alloc:7", -4)])
def test_injected_host_faults_are_reported_and_cleaned_up(monkeypatch, fault, code):
    """B200_INJECT_FAULT fakes a failing NCCL communicator set-up or the N-th
    device allocation on the host; b200_model_create returns B200_ENCCL /
    B200_ENOMEM, releases what it built, and the next model works."""
    import decode_model as M

    B = _B()
    cfg = M.LlamaConfig(n_layer=2, d_model=512, n_head=8, n_head_kv=2, head_dim=64, d_ff=1024, vocab=1024,
                        kv_size=64)
    monkeypatch.setenv("B200_INJECT_FAULT", fault)
    world = 2 if fault == "nccl_init" else 1
    nid = M.nccl_unique_id() if world == 2 else None
    with pytest.raises(B.B200Error) as ei:
        M.DecodeModel(cfg, tp_rank=0, tp_world=world, nccl_id=nid)
    assert ei.value.code == code
    monkeypatch.delenv("B200_INJECT_FAULT")
    free0 = torch.cuda.mem_get_info()[0]
    ok = M.DecodeModel(cfg)
    ok.init_synthetic(seed=1)
    ok.fill_kv_synthetic(seed=2, n_pos=8)
    assert 0 <= ok.decode(3, 8) < 1024
    ok.close()
    # nothing of the failed model is still held
    assert abs(torch.cuda.mem_get_info()[0] - free0) < (64 << 20)
    assert B.device_status(reset=True) == 0
