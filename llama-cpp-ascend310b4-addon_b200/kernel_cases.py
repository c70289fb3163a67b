"""Per-kernel cases of the decode path: timing and profiling driver.

    python kernel_cases.py                 # time every case, one JSON line each
    python kernel_cases.py gateup fa_l70   # time the named cases
    python kernel_cases.py --launches 3 gateup   # 3 plain launches (for a profiler)

Timing: each case is captured as a CUDA graph of 10 launches over rotating
copies of its weights / KV cache (together larger than the 126 MB L2, so
every launch reads HBM), replayed after warm-up, and timed with CUDA events
on the capturing stream.  GB/s counts algorithmic bytes: every weight (or
K/V) byte once, plus x and y.  Weights are random Q4_0/Q8_0 blocks with a
fixed small scale (the kernels' speed does not depend on the values).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import b200_decode as B  # noqa: E402

L2_BYTES = 126 << 20


def _torch():
    import torch

    return torch


def _blocks(wtype, n, k):
    torch = _torch()
    if wtype in (B.TYPE_F16, B.TYPE_A8W8):
        return (torch.randn(n, k, device="cuda") * 0.02).half()
    bb = B.BLOCK_BYTES[wtype]
    src = torch.randint(0, 255, (n, k // 32 * bb), dtype=torch.uint8, device="cuda")
    src.view(n, k // 32, bb)[:, :, 1] = 0x20  # f16 scale high byte: |d| ~ 2^-7
    return src


def _copies(nbytes, limit=64):
    return max(1, min(limit, math.ceil(2.5 * L2_BYTES / nbytes)))


# name: (weight type, N, K, q4 mode)
GEMV = {
    "config1_f16": (B.TYPE_F16, 8960, 1536, 0),
    # config 1's weight with M = 2 / 4 / 8 columns (the small-M branch)
    "config1_f16_m2": (B.TYPE_F16, 8960, 1536, 0),
    "config1_f16_m4": (B.TYPE_F16, 8960, 1536, 0),
    "config1_f16_m8": (B.TYPE_F16, 8960, 1536, 0),
    # a 4x wider k: one column (GEMV), four (one pass), eight (two passes)
    "wide_f16": (B.TYPE_F16, 8960, 6144, 0),
    "wide_f16_m4": (B.TYPE_F16, 8960, 6144, 0),
    "wide_f16_m8": (B.TYPE_F16, 8960, 6144, 0),
    "config3_q4_0": (B.TYPE_Q4_0, 1536, 8960, B.Q4_MODE_GGML),
    "config3_w4a16": (B.TYPE_Q4_0, 1536, 8960, B.Q4_MODE_W4A16),
    "config4_q8_0": (B.TYPE_Q8_0, 151936, 1536, 0),
    "config4_a8w8": (B.TYPE_A8W8, 151936, 1536, 0),  # the reference's per-token / per-column int8 scheme
    "gateup": (B.TYPE_Q4_0, 57344, 8192, B.Q4_MODE_GGML),  # Llama-3-70B gate+up rows
    "down": (B.TYPE_Q4_0, 8192, 28672, B.Q4_MODE_GGML),
    "qkv": (B.TYPE_Q4_0, 10240, 8192, B.Q4_MODE_GGML),
    "o": (B.TYPE_Q4_0, 8192, 8192, B.Q4_MODE_GGML),
    "lm_head": (B.TYPE_Q4_0, 128256, 8192, B.Q4_MODE_GGML),
}
# name: (n_head, n_head_kv, head_dim, n_kv, entry)
ATTN = {
    "fa_config2": (12, 2, 128, 4096, "workspace"),
    "fa_l70": (64, 8, 128, 4160, "workspace"),
    "fa_d256": (16, 4, 256, 4096, "workspace"),
    "fa_l70_static": (64, 8, 128, 4160, "static"),
}


def _row_bytes(wtype, k):
    if wtype == B.TYPE_A8W8:
        return k + 2  # int8 row + its f16 scale
    return 2 * k if wtype == B.TYPE_F16 else k // 32 * B.BLOCK_BYTES[wtype]


def gemv_case(name, reps_copies=None):
    torch = _torch()
    wtype, n, k, mode = GEMV[name]
    tail = name.rsplit("_m", 1)[-1]
    m = int(tail) if "_m" in name and tail.isdigit() else 1
    nbytes = n * _row_bytes(wtype, k) + m * (4 * k + 4 * n)
    copies = reps_copies or _copies(nbytes)
    src = _blocks(wtype, n, k)
    if wtype == B.TYPE_A8W8:
        ws = [B.a8w8_transform(src, n, k) for _ in range(copies)]
    else:
        ws = [B.repack(wtype, src, n, k) for _ in range(copies)]
    del src
    x = torch.randn(k, device="cuda") if m == 1 else torch.randn(m, k, device="cuda")
    y = torch.empty(n, device="cuda") if m == 1 else torch.empty(m, n, device="cuda")
    return (lambda i: B.mul_mat(ws[i % copies], x, y, q4_mode=mode)), nbytes


def attn_case(name, reps_copies=None):
    torch = _torch()
    hq, hkv, d, n_kv, entry = ATTN[name]
    kv_bytes = 2 * n_kv * hkv * d * 2
    nbytes = kv_bytes + 8 * hq * d
    copies = reps_copies or _copies(nbytes)
    q = torch.randn(hq, d, device="cuda")
    ks = [torch.randn(n_kv, hkv, d, device="cuda").half() for _ in range(copies)]
    vs = [torch.randn(n_kv, hkv, d, device="cuda").half() for _ in range(copies)]
    mask = torch.zeros(n_kv, device="cuda").half()
    out = torch.empty(hq, d, device="cuda")
    scale = d ** -0.5
    if entry == "static":
        return (lambda i: B.flash_attn_ext_static_scratch(q, ks[i % copies], vs[i % copies], mask, scale=scale,
                                                          out=out)), nbytes
    ws = B.fa_workspace(d, hq, hkv, n_kv, q.device)
    return (lambda i: B.flash_attn_ext(q, ks[i % copies], vs[i % copies], mask, scale=scale, out=out,
                                       workspace=ws)), nbytes


def make(name, copies=None):
    return gemv_case(name, copies) if name in GEMV else attn_case(name, copies)


def graph_time_us(fn, reps=20, inner=10):
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
    t = a.elapsed_time(b) * 1e3 / (reps * inner)
    del g
    return t


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("cases", nargs="*")
    ap.add_argument("--launches", type=int, default=0, help="run N plain launches of each case instead of timing")
    args = ap.parse_args()
    torch = _torch()
    names = args.cases or list(GEMV) + list(ATTN)
    for name in names:
        if name not in GEMV and name not in ATTN:
            raise SystemExit(f"unknown case {name}; known: {', '.join(list(GEMV) + list(ATTN))}")
    for name in names:
        if args.launches:
            fn, nbytes = make(name, copies=1)
            for i in range(args.launches):
                fn(i)
            torch.cuda.synchronize()
            print(json.dumps({"case": name, "launches": args.launches, "bytes": nbytes}), flush=True)
        else:
            fn, nbytes = make(name)
            t = graph_time_us(fn)
            print(json.dumps({"case": name, "us": round(t, 2), "bytes": nbytes, "GBs": round(nbytes / t / 1e3, 1)}),
                  flush=True)
        torch.cuda.empty_cache()
    st = B.device_status(reset=True)
    if st:
        raise SystemExit(f"device status {st:#x}")


if __name__ == "__main__":
    main()
