"""Benchmark of the GDN hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload: one recurrent decode step over 24 GDN
layers, B = 64 sequences per GPU, 32 value heads / 16 key heads, 128 x 128 fp32
state per head (6.44 GB of state per GPU), bf16 q/k/v/o.  A step is 24 launches
of the decode kernel, one per layer, each reading and writing its layer's state
once.  Work is sharded by batch: every GPU owns its own 64 sequences
(weak scaling, no collective on the data path).  `value` is the aggregate
algorithmic GB/s over all GPUs (bytes defined in orionsbelt_b200/metrics.py).
The state (6.44 GB per GPU) is far larger than L2 (126 MB), so no flush is
needed between steps.

Also reported on the same line: the chunkwise scan (config 2 shard: B = 8,
T = 32768, bf16 in / fp32 state) in tokens/s, `e2e` through the C ABI with the
step's inputs copied from pinned host memory and outputs copied back, the
roofline of the decode kernel, and the CPU baseline (the oracle port of the
reference's ref_delta_rule, OpenMP over (batch, head), on a bounded sample).

`--impl reference` times the reference path's CPU implementation of the same
decode step (the oracle port, all host threads) and prints the same metric;
under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from orionsbelt_b200 import metrics  # noqa: E402

METRIC = "GDN chunk-scan tokens/s & decode-step GB/s (% of HBM roofline) at 1/2/4/8 GPU"
CFG1 = dict(layers=24, B=64, Hk=16, Hv=32, dk=128, dv=128)
CFG2_SHARD = dict(B=8, T=32768, Hk=16, Hv=32, dk=128, dv=128)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-chunk", action="store_true", help="skip the chunk-scan measurement")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    return ap.parse_args()


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(n_gpus: int):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# --------------------------------------------------------------------- ours

def run_ours(args):
    import datetime

    import torch
    import torch.distributed as dist

    from orionsbelt_b200 import _lib, ops, synth

    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    L = _lib.lib()
    _lib.check(L.kai_gdn_cuda_set_device(local))
    peaks = load_peaks()
    c = CFG1
    bf16 = torch.bfloat16
    seed = 1000 + rank  # each rank owns different sequences

    # ---- per-layer inputs and states, resident in HBM
    layers = []
    for layer in range(c["layers"]):
        d = synth.device_gdn(c["B"], 1, c["Hk"], c["Hv"], c["dk"], c["dv"], g_scale=0.1, seed=seed * 100 + layer,
                             in_dtype=bf16, state_std=0.02)
        o = torch.empty((c["B"], c["Hv"], c["dv"]), dtype=bf16, device="cuda")
        args_l = ops.decode_args(d["S0"], d["q"][:, 0].contiguous(), d["k"][:, 0].contiguous(),
                                 d["v"][:, 0].contiguous(), d["g"][:, 0].contiguous(), d["beta"][:, 0].contiguous(),
                                 o, scale=1.0)
        layers.append((d, o, args_l))
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    launch = L.kai_run_gdn_delta_rule_decode_sm100a

    def step(events=None):
        for i, (_, _, a) in enumerate(layers):
            if events is not None:
                events[i][0].record(stream)
            rc = launch(a, sp)
            if rc:
                _lib.check(rc)
            if events is not None:
                events[i][1].record(stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()
    K = args.steps
    ev = [[[torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)] for _ in layers]
          for _ in range(K)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        t0.record(stream)
        for k in range(K):
            step(ev[k])
        t1.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = t0.elapsed_time(t1)
    launch_ms = [e[0].elapsed_time(e[1]) for row in ev for e in row]
    ms_max = ms
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = t.item()
    layer_bytes = metrics.decode_bytes(c["B"], c["Hk"], c["Hv"], c["dk"], c["dv"], e_state=4, e_in=2, e_out=2)
    step_bytes = layer_bytes * c["layers"]
    value = step_bytes * K * world / (ms_max / 1e3) / 1e9
    avg_launch_ms = sum(launch_ms) / len(launch_ms)
    achieved = layer_bytes / (avg_launch_ms / 1e3) / 1e9
    traffic = metrics.profiled_traffic(ROOT / "profiles", "decode_step_kernel")

    # ---- e2e through the C ABI: per-step inputs from pinned host memory, outputs back
    e2e = run_e2e_decode(args, layers, launch, sp, stream, world, barrier, step_bytes)

    # ---- chunk scan (config-2 shard) on this GPU
    chunk = None if args.no_chunk else run_chunk_bench(args, world, barrier, peaks)

    # ---- CPU baseline on a bounded sample (rank 0, N = 1 only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_decode_sample(seconds=10.0)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": K,
            "warmup": args.warmup,
            "ms_per_step": round(ms_max / K, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded N(0,1) q/k/v, L2-normalised q/k, sigmoid beta, -softplus*0.1 g, N(0,0.02) state)",
            "config": {
                "workload": "config 1: recurrent decode step over 24 GDN layers, batch 64 per GPU, 32 value / 16 key "
                            "heads, 128x128 fp32 state (6.44 GB per GPU), bf16 q/k/v/o",
                "global_batch": c["B"] * world, "layers": c["layers"], "heads_v": c["Hv"], "heads_k": c["Hk"],
                "head_dim": c["dk"], "state_dtype": "f32", "in_dtype": "bf16",
                "parallelism": f"batch shard x{world} (no collective)",
                "l2": "no flush needed: 6.44 GB of state per step per GPU >> 126 MB L2",
                "bytes_per_step_per_gpu": step_bytes,
            },
            "roofline": {
                "kernel": "decode_step_kernel<128, f32>",
                "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_src": peaks["src"],
                "traffic": traffic, "algorithmic_bytes_per_launch": layer_bytes,
                "avg_launch_us": round(avg_launch_ms * 1e3, 2),
            },
            "e2e": e2e,
            "gpu_launches": K * c["layers"],
            "clocks": clk.summary(),
            "chunk_scan": chunk,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_e2e_decode(args, layers, launch, sp, stream, world, barrier, step_bytes):
    """Decode step through the C ABI with host buffers: every step copies that
    step's q/k/v/g/beta for all 24 layers from pinned host memory into the
    device tensors the layer arguments point at (one packed copy), launches
    the 24 layers, and copies all 24 outputs back to pinned host memory.  The
    recurrent state stays resident in HBM between steps, as a decode engine
    keeps it."""
    import torch

    srcs = []
    for d, o, _ in layers:
        for key in ("q", "k", "v"):
            srcs.append(d[key])
        srcs.append(d["g"])
        srcs.append(d["beta"])
    nbytes = [t.numel() * t.element_size() for t in srcs]
    h2d = sum(nbytes)
    host_in = torch.empty(h2d, dtype=torch.uint8, pin_memory=True)
    dev_in = torch.empty(h2d, dtype=torch.uint8, device="cuda")
    off = 0
    for t, n in zip(srcs, nbytes):
        host_in[off:off + n].copy_(t.reshape(-1).view(torch.uint8).cpu())
        off += n
    outs = [o for _, o, _ in layers]
    d2h = sum(o.numel() * o.element_size() for o in outs)
    host_out = torch.empty(d2h, dtype=torch.uint8, pin_memory=True)
    dev_out = torch.empty(d2h, dtype=torch.uint8, device="cuda")

    def scatter_in():
        off = 0
        for t, n in zip(srcs, nbytes):
            t.reshape(-1).view(torch.uint8).copy_(dev_in[off:off + n], non_blocking=True)
            off += n

    def gather_out():
        off = 0
        for o in outs:
            n = o.numel() * o.element_size()
            dev_out[off:off + n].copy_(o.reshape(-1).view(torch.uint8), non_blocking=True)
            off += n

    def e2e_step():
        dev_in.copy_(host_in, non_blocking=True)
        scatter_in()
        for _, _, a in layers:
            launch(a, sp)
        gather_out()
        host_out.copy_(dev_out, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    t1.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = t0.elapsed_time(t1)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    return {"value": round(step_bytes * args.steps * world / (ms / 1e3) / 1e9, 1), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms / args.steps, 4)}


def run_chunk_bench(args, world, barrier, peaks):
    """Config-2 shard on this GPU: B=8, T=32768, bf16 q/k/v, fp32 state."""
    import torch

    from orionsbelt_b200 import _lib, ops, synth

    c = CFG2_SHARD
    d = synth.device_gdn(c["B"], c["T"], c["Hk"], c["Hv"], c["dk"], c["dv"], g_scale=0.1, seed=77,
                         in_dtype=torch.bfloat16)
    o = torch.empty_like(d["v"])
    S = d["S0"].clone()
    a = ops.chunk_args(d["q"], d["k"], d["v"], d["g"], d["beta"], S, o, scale=1.0)
    L = _lib.lib()
    stream = torch.cuda.current_stream()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    for _ in range(1):
        _lib.check(L.kai_run_gdn_chunk_delta_rule_sm100a(a, stream.cuda_stream))
    barrier()
    reps = max(1, min(args.steps, 3))
    tot = 0.0
    for _ in range(reps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        _lib.check(L.kai_run_gdn_chunk_delta_rule_sm100a(a, stream.cuda_stream))
        e1.record(stream)
        torch.cuda.synchronize()
        tot += e0.elapsed_time(e1)
    ms = tot / reps
    flops = metrics.chunk_flops(c["B"], c["T"], c["Hv"], c["dk"], 64)
    nbytes = metrics.chunk_bytes(c["B"], c["T"], c["Hk"], c["Hv"], c["dk"], c["dv"], e_in=2, e_out=2, e_state=4)
    tok = c["B"] * c["T"] * world / (ms / 1e3)
    return {"workload": "config 2 shard per GPU: B=8, T=32768, 16/32 heads, 128x128, bf16 q/k/v/o, fp32 state",
            "kernel": "chunk_scan_fp32_kernel (CUDA-core fp32)",
            "tokens_per_s": round(tok, 1), "ms": round(ms, 3),
            "tflops": round(flops / (ms / 1e3) / 1e12, 2), "gbs": round(nbytes / (ms / 1e3) / 1e9, 1),
            "tensor_frac_of_bf16_peak": round(flops / (ms / 1e3) / 1e12 / peaks["bf16_tflops"], 4),
            "hbm_frac": round(nbytes / (ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
            "l2": "256 MB buffer written before each timed call"}


def cpu_decode_sample(seconds: float = 10.0, nthreads: int = 0) -> dict:
    """Oracle port of ref_delta_rule (gpu/gdn_gpu_validate.c:100-118), OpenMP over
    (batch, head), on one config-1 layer at B=64, repeated for ~`seconds`."""
    import numpy as np

    import oracle
    from orionsbelt_b200 import synth

    orc, _ = oracle.require()
    c = CFG1
    r = np.random.default_rng(5)
    S = (r.standard_normal((c["B"], c["Hv"], c["dk"], c["dv"])) * 0.02).astype(np.float32)
    q = synth.l2norm(r.standard_normal((c["B"], c["Hk"], c["dk"])))
    k = synth.l2norm(r.standard_normal((c["B"], c["Hk"], c["dk"])))
    v = r.standard_normal((c["B"], c["Hv"], c["dv"])).astype(np.float32)
    beta = (1 / (1 + np.exp(-r.standard_normal((c["B"], c["Hv"]))))).astype(np.float32)
    g = (-synth.softplus(r.standard_normal((c["B"], c["Hv"]))) * 0.1).astype(np.float32)
    layer_bytes = metrics.decode_bytes(c["B"], c["Hk"], c["Hv"], c["dk"], c["dv"], e_state=4, e_in=4, e_out=4)
    orc.delta_rule_decode(S, q, k, v, g, beta, nthreads=nthreads)
    n, t_start = 0, time.perf_counter()
    while True:
        S, _ = orc.delta_rule_decode(S, q, k, v, g, beta, nthreads=nthreads)
        n += 1
        el = time.perf_counter() - t_start
        if el >= seconds:
            break
    cores = nthreads if nthreads > 0 else orc.num_threads()
    return {"value": round(layer_bytes * n / el / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{n} x one config-1 layer (B=64, 32 heads, 128x128 fp32 state, fp32 q/k/v), "
                      f"{el:.1f} s; oracle restatement of gpu/gdn_gpu_validate.c:100-118 (the reference's "
                      f"C decode step is in an OpenCL host file that does not build here)"}


# ---------------------------------------------------------------- reference

def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np

    import oracle
    from orionsbelt_b200 import synth

    orc, _ = oracle.require()
    c = CFG1
    r = np.random.default_rng(5)
    S = (r.standard_normal((c["B"], c["Hv"], c["dk"], c["dv"])) * 0.02).astype(np.float32)
    q = synth.l2norm(r.standard_normal((c["B"], c["Hk"], c["dk"])))
    k = synth.l2norm(r.standard_normal((c["B"], c["Hk"], c["dk"])))
    v = r.standard_normal((c["B"], c["Hv"], c["dv"])).astype(np.float32)
    beta = (1 / (1 + np.exp(-r.standard_normal((c["B"], c["Hv"]))))).astype(np.float32)
    g = (-synth.softplus(r.standard_normal((c["B"], c["Hv"]))) * 0.1).astype(np.float32)
    layer_bytes = metrics.decode_bytes(c["B"], c["Hk"], c["Hv"], c["dk"], c["dv"], e_state=4, e_in=4, e_out=4)
    for _ in range(args.warmup):
        S, _ = orc.delta_rule_decode(S, q, k, v, g, beta)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        S, _ = orc.delta_rule_decode(S, q, k, v, g, beta)
    el = time.perf_counter() - t0
    value = layer_bytes * args.steps / el / 1e9
    cores = orc.num_threads()
    sample = ("each step = one config-1 layer (B=64, 32 value heads, 128x128 fp32 state, fp32 q/k/v) of the "
              "24-layer decode step, on all host threads; oracle port of the reference's ref_delta_rule "
              "(gpu/gdn_gpu_validate.c:100-118; that file needs OpenCL headers and does not build here)")
    line = {"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config 1 decode step, one layer of 24 per step (CPU sample)", "global_batch": 64,
                       "parallelism": f"OpenMP x{cores} over (batch, head)"},
            "impl": "reference",
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
