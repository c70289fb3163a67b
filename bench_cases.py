"""Per-kernel benchmark cases of the decode path (``bench.py --case NAME``).

Each case is one hot kernel at one shape: the four single-kernel configs
(F16 GEMV 8960 x 1536, GQA decode attention 12/2 heads x 128 over 4096
positions, Q4_0 GEMV 1536 x 8960, Q8_0 x Q8_0 GEMV 151936 x 1536) and the
Llama-3-70B shapes of the decode step.  Two timings per case, both with CUDA
events on the launching stream after warm-up:

* ``exact``: the configured tensors, one launch per timed iteration, with
  the L2 flushed before every launch (a 256 MiB buffer written between
  launches, outside the timed events), so every launch reads HBM cold and
  pays its own launch and ramp-up -- the honest figure for working sets
  that would otherwise sit in the 126 MB L2;
* ``rotated``: a CUDA graph of 10 launches over rotating copies of the
  weights (or K/V cache) that together exceed the L2, timed per launch --
  the kernel's streaming rate with launch gaps hidden as in a decode step.

GB/s counts algorithmic bytes: every weight (or K/V) byte once plus the
activation in and the result out.  Weights are seeded N(0, 0.02^2) values
quantised with ggml's rules on the device; x ~ N(0, 1).
"""
from __future__ import annotations

import json
import math
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "llama-cpp-ascend310b4-addon_b200")
if PKG not in sys.path:
    sys.path.insert(0, PKG)

L2_BYTES = 126 << 20
FLUSH_BYTES = 256 << 20

# name: (weight type, N rows, K, q4 mode, columns M)
GEMV = {
    "config1": ("f16", 8960, 1536, 0, 1),
    "config3": ("q4_0", 1536, 8960, 0, 1),
    "config3_w4a16": ("q4_0", 1536, 8960, 1, 1),
    "config4": ("q8_0", 151936, 1536, 0, 1),
    "config4_a8w8": ("a8w8", 151936, 1536, 0, 1),  # the reference's own per-token / per-column int8 scheme
    "config1_m8": ("f16", 8960, 1536, 0, 8),        # the reference's small-M (M <= 8) NZ branch
    "gateup": ("q4_0", 57344, 8192, 0, 1),           # Llama-3-70B gate+up rows
    "down": ("q4_0", 8192, 28672, 0, 1),
    "qkv": ("q4_0", 10240, 8192, 0, 1),
    "o": ("q4_0", 8192, 8192, 0, 1),
    "lm_head": ("q4_0", 128256, 8192, 0, 1),
}
# name: (n_head, n_head_kv, head_dim, n_kv, entry)
ATTN = {
    "config2": (12, 2, 128, 4096, "workspace"),
    "fa_l70": (64, 8, 128, 4160, "workspace"),
    "fa_d256": (16, 4, 256, 4096, "workspace"),
    "fa_l70_static": (64, 8, 128, 4160, "static"),
}
# prefill MUL_MAT of an F16 weight on the tcgen05 tensor cores: (n rows, k, m tokens)
PREFILL = {
    "prefill_f16_512": (8192, 8192, 512),     # a Llama-70B-width projection over 512 prompt tokens
    "prefill_f16_128": (8960, 1536, 128),     # config 1's weight, 128 tokens
}
CASES = list(GEMV) + list(ATTN) + list(PREFILL)
KERNEL = {"f16": "gemv_kernel<FMT_F16>", "q4_0": "gemv_kernel<FMT_Q4>", "q8_0": "gemv_kernel<FMT_Q8>",
          "a8w8": "gemv_kernel<FMT_A8>"}


def _torch():
    import torch

    return torch


def _B():
    import b200_decode as B

    return B


def _wtype(name):
    B = _B()
    return {"f16": B.TYPE_F16, "q4_0": B.TYPE_Q4_0, "q8_0": B.TYPE_Q8_0, "a8w8": B.TYPE_A8W8}[name]


def _row_bytes(wt, k):
    if wt == "a8w8":
        return k + 2  # int8 row + its f16 scale
    return {"f16": 2 * k, "q4_0": k // 32 * 18, "q8_0": k // 32 * 34}[wt]


def _weights_ggml(wt, n, k, seed):
    """Seeded N(0, 0.02^2) weights on the device in ggml layout (F16 rows,
    or Q4_0 / Q8_0 blocks quantised with ggml's reference rules)."""
    torch = _torch()
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn(n, k, device="cuda", generator=g) * 0.02
    if wt in ("f16", "a8w8"):
        return w.half()
    x = w.view(n, k // 32, 32)
    amax_idx = x.abs().argmax(dim=2, keepdim=True)
    mx = torch.gather(x, 2, amax_idx)
    if wt == "q8_0":
        d = x.abs().amax(dim=2, keepdim=True) / 127.0
        idv = torch.where(d != 0, 1.0 / d, torch.zeros_like(d))
        q = torch.round(x * idv).clamp(-127, 127).to(torch.int8)
        blk = torch.empty(n, k // 32, 34, dtype=torch.uint8, device="cuda")
        blk[:, :, :2] = d.half().view(torch.uint8).view(n, k // 32, 2)
        blk[:, :, 2:] = q.view(torch.uint8)
        return blk.view(n, -1)
    d = mx / -8.0
    idv = torch.where(d != 0, 1.0 / d, torch.zeros_like(d))
    q = torch.clamp((x * idv + 8.5).to(torch.int8), max=15).to(torch.uint8)
    blk = torch.empty(n, k // 32, 18, dtype=torch.uint8, device="cuda")
    blk[:, :, :2] = d.half().view(torch.uint8).view(n, k // 32, 2)
    blk[:, :, 2:] = q[:, :, :16] | (q[:, :, 16:] << 4)
    return blk.view(n, -1)


def gemv_case(name, copies):
    torch = _torch()
    B = _B()
    wt, n, k, mode, m = GEMV[name]
    nbytes = n * _row_bytes(wt, k) + m * (4 * k + 4 * n)
    src = _weights_ggml(wt, n, k, seed=1234)
    code = _wtype(wt)
    if wt == "a8w8":
        ws = [B.a8w8_transform(src, n, k) for _ in range(copies)]
    else:
        ws = [B.repack(code, src, n, k) for _ in range(copies)]
    del src
    g = torch.Generator(device="cuda").manual_seed(99)
    x = torch.randn(k if m == 1 else (m, k), device="cuda", generator=g)
    y = torch.empty(n if m == 1 else (m, n), device="cuda")
    return (lambda i: B.mul_mat(ws[i % copies], x, y, q4_mode=mode)), nbytes


def attn_case(name, copies):
    torch = _torch()
    B = _B()
    hq, hkv, d, n_kv, entry = ATTN[name]
    nbytes = 2 * n_kv * hkv * d * 2 + 8 * hq * d + 2 * n_kv
    g = torch.Generator(device="cuda").manual_seed(7)
    q = torch.randn(hq, d, device="cuda", generator=g)
    ks = [torch.randn(n_kv, hkv, d, device="cuda", generator=g).half() for _ in range(copies)]
    vs = [torch.randn(n_kv, hkv, d, device="cuda", generator=g).half() for _ in range(copies)]
    mask = torch.zeros(n_kv, device="cuda").half()
    out = torch.empty(hq, d, device="cuda")
    scale = d ** -0.5
    if entry == "static":
        return (lambda i: B.flash_attn_ext_static_scratch(q, ks[i % copies], vs[i % copies], mask, scale=scale,
                                                          out=out)), nbytes
    ws = B.fa_workspace(d, hq, hkv, n_kv, q.device)
    return (lambda i: B.flash_attn_ext(q, ks[i % copies], vs[i % copies], mask, scale=scale, out=out,
                                       workspace=ws)), nbytes


def prefill_case(name, copies):
    torch = _torch()
    B = _B()
    n, k, m = PREFILL[name]
    g = torch.Generator(device="cuda").manual_seed(5)
    ws = [(torch.randn(n, k, device="cuda", generator=g) * 0.02).half() for _ in range(copies)]
    x = torch.randn(m, k, device="cuda", generator=g)
    y = torch.empty(m, n, device="cuda")
    B.mul_mat_f16_tc(ws[0], x, n, k, y)  # sizes the cached workspace outside any capture
    return (lambda i: B.mul_mat_f16_tc(ws[i % copies], x, n, k, y)), n * k * 2 + m * k * 4 + m * n * 4


def make(name, copies=1):
    if name in PREFILL:
        return prefill_case(name, copies)
    return gemv_case(name, copies) if name in GEMV else attn_case(name, copies)


def prefill_line(name, peak_tflops, peak_kind):
    """Tensor-core roofline of the prefill GEMM: 2 n k m flops per launch
    over the CUDA-event time of rotated launches (weights > L2)."""
    torch = _torch()
    B = _B()
    n, k, m = PREFILL[name]
    copies = max(1, min(16, math.ceil(2.5 * L2_BYTES / (n * k * 2))))
    fn, nbytes = prefill_case(name, copies)
    us = time_rotated(fn, copies)
    del fn
    torch.cuda.empty_cache()
    st = B.device_status(reset=True)
    if st:
        raise SystemExit(f"device status {st:#x} after case {name}")
    tflops = 2.0 * n * k * m / (us * 1e-6) / 1e12
    return {
        "metric": f"{name}: achieved dense f16 TFLOP/s", "case": name, "value": tflops, "unit": "TFLOP/s",
        "higher_is_better": True, "n_gpus": 1, "data": "synthetic (seeded N(0,0.02^2) weights, N(0,1) x)",
        "config": {"workload": name, "n": n, "k": k, "m": m, "weight": "f16",
                   "l2": "rotated weight copies larger than L2"},
        "us_rotated": us,
        "roofline": {"bound": "tensor", "kernel": "gemm_f16_tc_kernel (tcgen05.mma kind::f16, TMEM accumulators)",
                     "flops_per_launch": 2 * n * k * m, "achieved": tflops, "peak": peak_tflops, "unit": "TFLOP/s",
                     "peak_source": peak_kind, "frac": tflops / peak_tflops,
                     "hbm_bytes_per_launch": nbytes},
    }


def case_bytes(name):
    if name in GEMV:
        wt, n, k, _, m = GEMV[name]
        return n * _row_bytes(wt, k) + m * (4 * k + 4 * n)
    hq, hkv, d, n_kv, _ = ATTN[name]
    return 2 * n_kv * hkv * d * 2 + 8 * hq * d + 2 * n_kv


def rotated_copies(name):
    return max(1, min(64, math.ceil(2.5 * L2_BYTES / case_bytes(name))))


def time_rotated(fn, copies, reps=20, inner=10):
    """us per launch: a graph of `inner` launches over rotating copies."""
    torch = _torch()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for i in range(3):
            fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(inner):
            fn(i)
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        for _ in range(3):
            g.replay()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s)
        for _ in range(reps):
            g.replay()
        b.record(s)
    torch.cuda.synchronize()
    del g
    return a.elapsed_time(b) * 1e3 / (reps * inner)


def time_flushed(fn, reps=50, warmup=5):
    """Median us of single launches, each after an L2 flush outside the
    events: a 256 MiB buffer is read (summed), which evicts the case's lines
    and leaves only clean ones; a write-based flush would leave ~126 MB of
    dirty lines that the timed launch then has to write back."""
    torch = _torch()
    s = torch.cuda.current_stream()
    flush = torch.ones(FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    sink = torch.empty(1, dtype=torch.float32, device="cuda")
    ts = []
    for it in range(warmup + reps):
        torch.sum(flush, dim=0, keepdim=True, out=sink)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s)
        fn(0)
        b.record(s)
        b.synchronize()
        if it >= warmup:
            ts.append(a.elapsed_time(b) * 1e3)
    return statistics.median(ts)


def cpu_case(name, reps=20):
    """The CPU oracle (C restatement of ggml-cpu, OpenMP over every host
    core) on the same shape: median seconds per call and the thread count."""
    import numpy as np

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    O.build()
    r = np.random.default_rng(5)
    if name in GEMV:
        wt, n, k, mode, m = GEMV[name]
        if wt not in ("f16", "q4_0", "q8_0") or m != 1:
            return None
        x = r.standard_normal(k).astype(np.float32)
        if wt == "f16":
            w = (r.standard_normal((n, k)) * 0.02).astype(np.float16)
            fn = lambda: O.mul_mat_f16(w, x)  # noqa: E731
        elif wt == "q4_0":
            w = O.synth_q4_0(11, 0.02, 0, n, k)
            fn = lambda: O.mul_mat_q4_0(w, x, mode)  # noqa: E731
        else:
            w = O.quantize_q8_0((r.standard_normal((n, k)) * 0.02).astype(np.float32))
            fn = lambda: O.mul_mat_q8_0(w, x)  # noqa: E731
    else:
        hq, hkv, d, n_kv, _ = ATTN[name]
        q = r.standard_normal((hq, d)).astype(np.float32)
        kk = r.standard_normal((n_kv, hkv, d)).astype(np.float16)
        vv = r.standard_normal((n_kv, hkv, d)).astype(np.float16)
        fn = lambda: O.flash_attn_decode(q, kk, vv, None, mode=1)  # noqa: E731
    fn()
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts), os.cpu_count() or 1


def case_line(name, peak, peak_kind, with_cpu=True):
    """One JSON-ready dict for the case (both timings, roofline, CPU)."""
    torch = _torch()
    B = _B()
    nbytes = case_bytes(name)
    fn, _ = make(name, copies=1)
    us_exact = time_flushed(fn)
    del fn
    torch.cuda.empty_cache()
    copies = rotated_copies(name)
    fn, _ = make(name, copies=copies)
    us_rot = time_rotated(fn, copies)
    del fn
    torch.cuda.empty_cache()
    st = B.device_status(reset=True)
    if st:
        raise SystemExit(f"device status {st:#x} after case {name}")
    gbs_exact = nbytes / (us_exact * 1e-6) / 1e9
    gbs_rot = nbytes / (us_rot * 1e-6) / 1e9
    if name in GEMV:
        wt, n, k, mode, m = GEMV[name]
        kern = "gemm_small_m_kernel" if m > 1 else KERNEL[wt] + (" (W4A16 mode)" if mode == 1 else "")
        shape = {"n": n, "k": k, "m": m, "weight": wt}
    else:
        hq, hkv, d, n_kv, entry = ATTN[name]
        kern = ("fa_decode_kernel (static scratch)" if entry == "static" else
                "fa_mma_kernel" if d in (64, 128) else "fa_decode_kernel")
        shape = {"n_head": hq, "n_head_kv": hkv, "head_dim": d, "n_kv": n_kv}
    line = {
        "metric": f"{name}: achieved HBM GB/s", "case": name, "value": gbs_exact, "unit": "GB/s",
        "higher_is_better": True, "n_gpus": 1, "data": "synthetic (seeded N(0,0.02^2) weights, N(0,1) x / KV)",
        "config": dict(workload=name, **shape, l2="exact: flushed before every launch; rotated: copies > L2"),
        "us_exact_l2_flushed": us_exact, "us_rotated": us_rot,
        "roofline": {"bound": "hbm", "kernel": kern, "bytes_per_launch": nbytes, "peak": peak, "unit": "GB/s",
                     "peak_source": peak_kind, "achieved": gbs_exact, "frac": gbs_exact / peak,
                     "achieved_rotated": gbs_rot, "frac_rotated": gbs_rot / peak},
    }
    if with_cpu:
        c = cpu_case(name)
        if c is not None:
            sec, cores = c
            line["cpu_baseline"] = {"value": nbytes / sec / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
                                    "sample": "the CPU oracle on the same shape, median of 20 calls",
                                    "us_per_call": sec * 1e6}
    return line


def run_launches(name, n):
    """n plain launches of the case (for a profiler's launch list)."""
    torch = _torch()
    fn, nbytes = make(name, copies=1)
    for i in range(n):
        fn(i)
    torch.cuda.synchronize()
    print(json.dumps({"case": name, "launches": n, "bytes": nbytes}), flush=True)
