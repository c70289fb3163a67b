"""Benchmark: batch-1 greedy decode of the Llama-3-70B-shaped Q4_0 model
(80 layers, Q4_0 weights, KV cache prefilled to 4096 positions) on N B200s
of one node, tensor parallel.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python bench.py --case NAME [--launches L]     # one kernel (bench_cases.py)

N > 1 is launched one process per GPU with torch.distributed.run.  A step is
one decode token: the whole captured CUDA graph (80 layers + lm_head + argmax,
NCCL all-reduces at N > 1) with the argmax fed back on the device.  Weights
are random-init Q4_0 from N(0, 0.02^2) (synthetic, no checkpoint); the KV
cache is prefilled with seeded N(0, 1) f16 for 4096 positions.  Timed with
CUDA events on the model stream between barriers + synchronisations, max over
ranks.  Prints one JSON line on rank 0.

--impl reference times the CPU oracle (oracle/refcpu.c, a C restatement of
ggml-cpu's decode semantics; the reference add-on's own kernels need an
Ascend NPU and llama.cpp's CPU backend is not in this image) on the host
cores over whole 80-layer greedy tokens of the same model: the same seeded
weights and KV prefill, regenerated on the host bit for bit.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(ROOT, "llama-cpp-ascend310b4-addon_b200"), os.path.join(ROOT, "oracle")]

METRIC = "batch-1 decode tok/s (Llama-3-70B-shape Q4_0, KV 4096, greedy)"
UNIT = "tok/s"
N_PREFILL = 4096
SEED = 20261201


def model_cfg(steps_total: int):
    import decode_model as M

    kv = N_PREFILL + max(128, steps_total + 2)
    return M.LlamaConfig(kv_size=kv, **M.LLAMA3_70B)


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def measured_tensor_peak():
    """Dense bf16/f16 tensor peak (burst: the prefill GEMM is timed alone)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def ncu_traffic():
    """Per-launch DRAM bytes of the gate/up GEMV from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "gemv_q4_0_gateup_traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return None


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def mark(self):
        """Start of the timed region: later readings are the region's."""
        self.first = len(self.lines)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.lines = self.lines[getattr(self, "first", 0):]
        if not self.lines:
            # region shorter than the sampling period: one reading right at its end
            try:
                r = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                    "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=10)
                self.lines.extend(x.strip() for x in r.stdout.splitlines() if x.strip())
            except Exception:
                pass
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for i, n in enumerate(names):
                if f[5 + i].lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ CPU side

def host_mem_available() -> int:
    try:
        with open("/proc/meminfo") as f:
            for ln in f:
                if ln.startswith("MemAvailable:"):
                    return int(ln.split()[1]) * 1024
    except OSError:
        pass
    return 0


class CpuModel:
    """The CPU oracle (oracle/refcpu.c: ggml-cpu's decode semantics restated
    in C, OpenMP over every host core) holding the same synthetic model as
    the GPU arm: the first `layers` layers of the Llama-3-70B shape (all 80
    for the reference arm), the same seeded Q4_0 weights and KV prefill,
    regenerated on the host bit for bit (oracle.synth_llama_weights)."""

    def __init__(self, layers: int, n_tokens: int):
        import decode_model as M
        import oracle as O

        O.build()
        cfg = model_cfg(n_tokens)
        cfg.n_layer = layers
        c = cfg.as_dict()
        self.layers = layers
        W = O.synth_llama_weights(c, SEED, 0.02)
        kc, vc = O.synth_llama_kv(c, SEED + 1, N_PREFILL)
        self.ref = O.OracleLlama(c, W, kc, vc)
        self.cores = os.cpu_count() or 1
        self.tok, self.pos = 128000, N_PREFILL

    def step(self, l0=0, l1=None, head=True) -> float:
        """Layers [l0, l1) of the current greedy token (the embedding when
        l0 == 0) and, with head, the lm_head + argmax that ends the token;
        returns seconds."""
        t0 = time.perf_counter()
        nxt = self.ref.step(self.tok, self.pos, l0=l0, l1=l1, do_head=head)
        t = time.perf_counter() - t0
        if head:
            self.tok, self.pos = nxt, self.pos + 1
        return t

    def sampled_token(self):
        """(seconds of the sampled layers, seconds of the lm_head) of one token."""
        t_layers = self.step(0, self.layers, head=False)
        t_head = self.step(self.layers, self.layers, head=True)
        return t_layers, t_head


def cpu_baseline(tokens: int = 3):
    """Bounded CPU sample for the GPU arm's line: 2 of the 80 layers plus the
    lm_head per token (same weights as the GPU arm's first layers), tok/s
    extrapolated to 80 layers."""
    cm = CpuModel(layers=2, n_tokens=tokens + 2)
    cm.sampled_token()
    vals = []
    for _ in range(tokens):
        t_layers, t_head = cm.sampled_token()
        vals.append(1.0 / (80 * t_layers / 2 + t_head))
    sample = (f"2 of 80 layers at full width + lm_head per token, the GPU arm's weights and KV, "
              f"timed per token and extrapolated (80 x layer time + head time), median of {tokens} tokens")
    return statistics.median(vals), cm.cores, sample


def bench_config(world: int, steps: int) -> dict:
    """The workload description both arms print (identical for the same N, K)."""
    return {"workload": "Llama-3-70B-shape Q4_0 batch-1 greedy decode, KV prefilled 4096",
            "model": "llama3-70b-shape (80L, d8192, 64/8 heads, ffn 28672, vocab 128256)",
            "global_batch": 1, "seq_len": N_PREFILL + steps // 2, "prefill": N_PREFILL,
            "parallelism": f"tp{world}",
            "data_seed": SEED}


DATA = "synthetic (seeded N(0,0.02^2) weights quantised to Q4_0; KV prefilled N(0,1) f16; same bytes in both arms)"


# --------------------------------------------------------------------- arms

def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    return world, rank, local


def run_reference(args):
    """The reference arm: the CPU oracle on the host cores timing whole
    80-layer greedy tokens of the same model (weights, KV prefill, start
    token and positions as the GPU arm).  Rank 0 only."""
    world, rank, _ = dist_setup(args.gpus)
    if rank != 0:
        return
    need = 44 << 30  # 39.5 GB of Q4_0 weights + KV cache + working set
    avail = host_mem_available()
    total = args.warmup + args.steps
    if avail and avail < need:
        # not enough host memory for the whole model: time a bounded sample
        cm = CpuModel(layers=2, n_tokens=total + 2)
        tl, th = [], []
        for i in range(total):
            a, b = cm.sampled_token()
            if i >= args.warmup:
                tl.append(a)
                th.append(b)
        per_step = statistics.mean(tl) + statistics.mean(th)
        value = 1.0 / (80 * statistics.mean(tl) / 2 + statistics.mean(th))
        sample = (f"host memory {avail >> 30} GiB < {need >> 30} GiB: each step times 2 of the 80 layers + the "
                  "lm_head (ms_per_step); value extrapolated to 80 layers")
        extrapolated = True
    else:
        cm = CpuModel(layers=80, n_tokens=total + 2)
        for _ in range(args.warmup):
            cm.step()
        ts = [cm.step() for _ in range(args.steps)]
        per_step = statistics.mean(ts)
        value = len(ts) / sum(ts)
        sample = "whole 80-layer greedy tokens (embedding, 80 layers, lm_head, argmax), every step timed"
        extrapolated = False
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per_step * 1000.0, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "q4_0xq8_0 int32 dots, fp32", "data": DATA,
        "config": bench_config(args.gpus, args.steps),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cm.cores, "kind": "port", "sample": sample,
                         "extrapolated": extrapolated},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "CPU oracle (C restatement of ggml-cpu decode semantics, OpenMP over all host cores); the "
                "reference add-on runs on an Ascend NPU and llama.cpp's CPU backend is absent from this image",
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    import torch.distributed as dist

    import decode_model as M

    world, rank, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=120))
    nid = None
    if world > 1:
        obj = [M.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nid = obj[0]
    total = args.warmup + args.steps
    cfg = model_cfg(total)
    m = M.DecodeModel(cfg, device=local, tp_rank=rank, tp_world=world, nccl_id=nid)
    m.init_synthetic(seed=SEED, sigma=0.02)
    m.fill_kv_synthetic(seed=SEED + 1, n_pos=N_PREFILL)
    m.capture()
    stream = torch.cuda.ExternalStream(m.stream_handle(), device=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-resident steps (graph replay, token fed back on the GPU)
    m.set_state(128000, N_PREFILL, advance=True)
    clocks = ClockSampler(local)
    clocks.start()  # running (under load) before the timed region starts
    for _ in range(args.warmup):
        m.launch()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clocks.mark()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        m.launch()
    ev1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    barrier()
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    tok_s = args.steps / (ms / 1000.0)

    # ---- end to end through the public decode call (host token in/out)
    tok = 128000
    pos0 = N_PREFILL
    for i in range(2):
        tok = m.decode(tok, pos0 + i)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(args.steps):
        tok = m.decode(tok, pos0 + 2 + i)
    t1 = time.perf_counter()
    e2e_s = t1 - t0
    if world > 1:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = args.steps / e2e_s

    # ---- dominant kernel: gate/up GEMV.  Per-launch time from CUDA events
    # around a graph of the step's 80 gate/up launches (each layer's own
    # weights, so nothing is served from L2); the eager per-class pass below
    # (events around every kernel, no launch overlap) gives the breakdown.
    m.set_state(128000, N_PREFILL, advance=True)
    gu_us = m.time_gate_up(iters=5)
    prof = m.profile(iters=2)
    # where a captured step's time goes, measured inside the step (device
    # clock stamps at each kernel's start and end; the classes add up to it)
    m.set_state(128000, N_PREFILL, advance=True)
    m.timeline()
    tl = m.timeline()
    d, ff_l = cfg.d_model, cfg.d_ff // world
    gu_bytes = 2 * ff_l * (d // 32) * 18 + d * 4 * 2  # Q4_0 weights + x + ffn_norm
    peak, peak_kind = measured_peaks()
    achieved = gu_bytes / (gu_us * 1e-6) / 1e9
    tr = ncu_traffic()
    traffic = None
    if tr and int(tr.get("tp", 1)) == world:
        traffic = tr.get("dram_bytes_per_launch")
    ctx_mid = N_PREFILL + args.steps // 2
    step_bytes = m.step_bytes(ctx_mid)
    if world > 1:
        barrier()
    if rank == 0:
        # embed, 5 per layer (qkv, attention, o, gate/up, down), lm_head, finish; at
        # tp > 1 the default mode adds our all-reduce kernel after o and down (the
        # argmax all-reduce is NCCL's; B200_TP_ALLREDUCE=nccl or fused launch none of ours)
        launches_per_step = 1 + 5 * cfg.n_layer + 1 + 1
        if world > 1 and os.environ.get("B200_TP_ALLREDUCE", "") not in ("nccl", "fused"):
            launches_per_step += 2 * cfg.n_layer
        cpu_v, cores, sample = (None, None, None)
        if world == 1 and not args.no_cpu:
            cpu_v, cores, sample = cpu_baseline()
        line = {
            "metric": METRIC, "value": tok_s, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "q4_0xq8_0 int32 dots, fp32", "data": DATA,
            "config": bench_config(world, args.steps),
            "l2": "no flush needed: each step streams %.1f GB of weights per GPU (> 126 MB L2)" % (step_bytes / 1e9),
            "roofline": {"bound": "hbm", "kernel": "gemv_q4_0 gate/up (fused RMSNorm+Q8_0+SwiGLU)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": peak_kind, "traffic": traffic,
                         "bytes_per_launch": gu_bytes, "us_per_launch": gu_us,
                         "us_per_launch_eager": prof["gate_up"],
                         "step_bytes": step_bytes,
                         "step_frac": step_bytes / (ms / args.steps * 1e-3) / 1e9 / peak},
            "kernel_us": prof,
            "step_breakdown_us": {"step": tl["step_us"], "advance": tl["advance_us"], "span": tl["span_us"],
                                  "phases": tl["phases_us"]},
            "clocks": clk,
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": 16, "d2h_bytes_per_step": 4},
            "gpu_launches": launches_per_step * args.steps,
        }
        if cpu_v is not None:
            line["cpu_baseline"] = {"value": cpu_v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample,
                                    "extrapolated": True}
        print(json.dumps(line), flush=True)
    m.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_case(args):
    """One JSON line per kernel case: L2-flushed exact-config and rotated
    (copies larger than L2) timings, roofline fraction, CPU oracle beside."""
    import torch

    import bench_cases as BC

    names = BC.CASES if args.case == "all" else [args.case]
    for n in names:
        if n not in BC.CASES:
            raise SystemExit(f"unknown case {n}; known: {', '.join(BC.CASES)}")
    torch.cuda.set_device(0)
    if args.launches:
        for n in names:
            BC.run_launches(n, args.launches)
        return
    peak, kind = measured_peaks()
    tpeak, tkind = measured_tensor_peak()
    for n in names:
        clocks = ClockSampler(0)
        clocks.start()
        if n in BC.PREFILL:
            line = BC.prefill_line(n, tpeak, tkind)
        else:
            line = BC.case_line(n, peak, kind, with_cpu=not args.no_cpu)
        line["clocks"] = clocks.stop()
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline sample")
    ap.add_argument("--case", default=None,
                    help="one kernel case instead of the decode step (bench_cases.CASES, or 'all')")
    ap.add_argument("--launches", type=int, default=0, help="with --case: only run L plain launches (profilers)")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.case is not None:
        run_case(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
