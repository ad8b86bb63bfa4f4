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

import numpy as np

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
    ap.add_argument("--no-rows", action="store_true", help="skip the per-row measurements")
    ap.add_argument("--no-model", action="store_true", help="skip the config-4 model decode")
    return ap.parse_args()


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


class ClockSampler:
    """SM clocks and throttle reasons sampled during the timed region.

    A thread polls NVML (read-only queries) every 2 ms, so a timed region of a
    few milliseconds still holds several samples; it is started, and has taken
    its first sample, before the region begins.  Without NVML the recipe's
    `nvidia-smi -lms 200` line is used instead (which a region this short may
    fall between)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.thread = None
        self.samples = []  # (sm MHz, max MHz, set of reason names)
        self.source = None

    def _nvml_handle(self, nv):
        import torch

        props = torch.cuda.get_device_properties(self.index)
        try:
            return nv.nvmlDeviceGetHandleByUUID("GPU-" + str(props.uuid))
        except Exception:
            pass
        try:
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            return nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.index)

    def _start_nvml(self) -> bool:
        import threading

        try:
            import pynvml as nv

            nv.nvmlInit()
            h = self._nvml_handle(nv)
            mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        except Exception:
            return False
        bits = [nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap]
        self.stop = threading.Event()
        first = threading.Event()

        def poll():
            while True:
                try:
                    sm = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((sm, mx, {n for n, b in zip(self.NAMES, bits) if r & b}))
                except Exception:
                    pass
                first.set()
                if self.stop.wait(0.002):
                    break

        self.thread = threading.Thread(target=poll, daemon=True)
        self.thread.start()
        first.wait(2.0)
        self.source = "nvml, 2 ms"
        return True

    def __enter__(self):
        if self._start_nvml():
            return self
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.source = "nvidia-smi, 200 ms"
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
            return
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            for ln in out.splitlines():
                f = [x.strip() for x in ln.split(",")]
                if len(f) < 9:
                    continue
                try:
                    sm, mx = float(f[1]), float(f[2])
                except ValueError:
                    continue
                self.samples.append((sm, mx, {n for n, v in zip(self.NAMES, f[5:9]) if v.lower() == "active"}))

    def summary(self) -> dict:
        sm = [x[0] for x in self.samples]
        reasons = set().union(*[x[2] for x in self.samples]) if self.samples else set()
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": self.samples[-1][1] if self.samples else None, "reasons": sorted(reasons),
                "samples": len(sm), "source": self.source}


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
    from orionsbelt_b200 import shard
    seed = shard.rank_seed(1, rank)  # each rank owns its own 64 sequences (weak scaling)

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
    launch = L.kai_run_gdn_delta_rule_decode_sm100a

    def launch_layers(arg_list):
        sp = torch.cuda.current_stream().cuda_stream
        for a in arg_list:
            rc = launch(a, sp)
            if rc:
                _lib.check(rc)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # One step = 24 layer launches, captured once into a CUDA graph so the
    # timed loop measures the GPU, not Python's launch rate.
    launch_layers([a for _, _, a in layers])  # eager warm-up before capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        launch_layers([a for _, _, a in layers])
    for _ in range(args.warmup):
        graph.replay()
    barrier()
    K = args.steps
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(K + 1)]
    with ClockSampler(local) as clk:
        ev[0].record(stream)
        for k in range(K):
            graph.replay()
            ev[k + 1].record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = ev[0].elapsed_time(ev[K])
    step_ms = [ev[k].elapsed_time(ev[k + 1]) for k in range(K)]
    ms_max = ms
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = t.item()
    layer_bytes = metrics.decode_bytes(c["B"], c["Hk"], c["Hv"], c["dk"], c["dv"], e_state=4, e_in=2, e_out=2)
    step_bytes = layer_bytes * c["layers"]
    value = step_bytes * K * world / (ms_max / 1e3) / 1e9
    # Average launch duration of the decode kernel: step time / 24 launches
    # (back-to-back graph nodes, so inter-launch gaps count against it).
    avg_launch_ms = statistics.median(step_ms) / c["layers"]
    achieved = layer_bytes / (avg_launch_ms / 1e3) / 1e9
    traffic = metrics.profiled_traffic(ROOT / "profiles", "decode_step_kernel")

    # ---- e2e through the C ABI: per-step inputs from pinned host memory, outputs back
    del graph
    e2e = run_e2e_decode(args, layers, launch_layers, world, barrier, step_bytes)

    # ---- chunk scan (config-2 shard) on this GPU
    chunk = None if args.no_chunk else run_chunk_bench(args, world, barrier, peaks, seed)

    # ---- strong scaling: the fixed global problems split over the ranks
    strong = run_strong(args, world, rank, barrier, peaks)

    # ---- config 4: the hybrid model's decode, tensor-parallel over the ranks
    model = None if args.no_model else run_model(args, world, rank, barrier, peaks)

    # ---- every other hot-path row on its own configuration (this GPU)
    rows = None if (args.no_rows or world > 1) else run_rows(args, peaks)

    # ---- CPU baselines on bounded samples (rank 0, N = 1 only): the headline
    # decode step, and one per row beside its GPU figure
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        nthreads = host_threads()
        cpu = cpu_decode_sample(seconds=5.0, nthreads=nthreads)
        crow = cpu_rows(nthreads)
        if rows is not None:
            for name, row in rows.items():
                if name in crow:
                    row["cpu_baseline"] = crow[name]
        if chunk is not None and "chunk_cfg2" in crow:
            chunk["cpu_baseline"] = crow["chunk_cfg2"]

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
            "strong_scaling": strong,
            "model_config4": model,
            "rows": rows,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_e2e_decode(args, layers, launch_layers, world, barrier, step_bytes):
    """Decode step through the C ABI with host buffers.  Every step copies that
    step's q/k/v/g/beta for all 24 layers from pinned host memory to the GPU
    (one packed copy), runs the 24 layer launches, and copies the 24 outputs
    back to pinned host memory; the recurrent state stays resident in HBM, as
    a decode engine keeps it.  Two input/output buffer sets let step k+1's
    upload and step k-1's download run on copy streams while step k computes."""
    import torch

    from orionsbelt_b200 import ops

    c = CFG1
    B, Hk, Hv, dk, dv = c["B"], c["Hk"], c["Hv"], c["dk"], c["dv"]
    per_layer = [("q", (B, Hk, dk), torch.bfloat16), ("k", (B, Hk, dk), torch.bfloat16),
                 ("v", (B, Hv, dv), torch.bfloat16), ("g", (B, Hv), torch.float32), ("beta", (B, Hv), torch.float32)]
    in_bytes = sum(torch.Size(sh).numel() * torch.empty(0, dtype=dt).element_size() for _, sh, dt in per_layer)
    out_bytes = B * Hv * dv * 2
    h2d, d2h = in_bytes * len(layers), out_bytes * len(layers)

    def views(buf, layer, spec, base):
        off = base + layer * sum(torch.Size(sh).numel() * torch.empty(0, dtype=dt).element_size() for _, sh, dt in spec)
        out = {}
        for name, sh, dt in spec:
            n = torch.Size(sh).numel() * torch.empty(0, dtype=dt).element_size()
            out[name] = buf[off:off + n].view(dt).view(sh)
            off += n
        return out

    # Pinned buffers are first touched on the CPUs of the GPU's NUMA node (the
    # process affinity is narrowed for the allocation and restored after).
    numa = gpu_numa_node(torch.cuda.current_device())
    saved_aff = None
    if numa["cpus"]:
        try:
            saved_aff = os.sched_getaffinity(0)
            os.sched_setaffinity(0, numa["cpus"])
        except (AttributeError, OSError):
            saved_aff = None
    sets = []
    for b in range(2):
        host_in = torch.empty(h2d, dtype=torch.uint8, pin_memory=True)
        dev_in = torch.empty(h2d, dtype=torch.uint8, device="cuda")
        host_out = torch.empty(d2h, dtype=torch.uint8, pin_memory=True)
        dev_out = torch.empty(d2h, dtype=torch.uint8, device="cuda")
        arg_list = []
        for li, (d, _, _) in enumerate(layers):
            vi = views(dev_in, li, per_layer, 0)
            vi["q"].copy_(d["q"][:, 0])
            vi["k"].copy_(d["k"][:, 0])
            vi["v"].copy_(d["v"][:, 0])
            vi["g"].copy_(d["g"][:, 0])
            vi["beta"].copy_(d["beta"][:, 0])
            o = dev_out[li * out_bytes:(li + 1) * out_bytes].view(torch.bfloat16).view(B, Hv, dv)
            arg_list.append(ops.decode_args(d["S0"], vi["q"], vi["k"], vi["v"], vi["g"], vi["beta"], o, scale=1.0))
        torch.cuda.synchronize()
        host_in.copy_(dev_in)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            launch_layers(arg_list)
        sets.append(dict(host_in=host_in, dev_in=dev_in, host_out=host_out, dev_out=dev_out, graph=g,
                         args=arg_list))
    if saved_aff is not None:
        os.sched_setaffinity(0, saved_aff)
    compute = torch.cuda.current_stream()
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    done = [torch.cuda.Event(), torch.cuda.Event()]
    uploaded = [torch.cuda.Event(), torch.cuda.Event()]
    downloaded = [torch.cuda.Event(), torch.cuda.Event()]

    def upload(k):
        st = sets[k % 2]
        with torch.cuda.stream(up):
            up.wait_event(downloaded[k % 2]) if k >= 2 else None
            up.wait_event(done[k % 2]) if k >= 2 else None
            st["dev_in"].copy_(st["host_in"], non_blocking=True)
            uploaded[k % 2].record(up)

    def run(n, t0=None, t1=None):
        if t0 is not None:
            t0.record(up)
        upload(0)
        for k in range(n):
            if k + 1 < n:
                upload(k + 1)
            st = sets[k % 2]
            compute.wait_event(uploaded[k % 2])
            st["graph"].replay()
            done[k % 2].record(compute)
            with torch.cuda.stream(down):
                down.wait_event(done[k % 2])
                st["host_out"].copy_(st["dev_out"], non_blocking=True)
                downloaded[k % 2].record(down)
        if t1 is not None:
            t1.record(down)

    run(args.warmup)
    torch.cuda.synchronize()
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    run(args.steps, t0, t1)
    torch.cuda.synchronize()
    barrier()
    ms = t0.elapsed_time(t1)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    for st in sets:
        del st["graph"]
    # The host copies alone, each timed on its own stream (max over ranks):
    # the per-rank and aggregate host-link rates that bound this leg.
    copies = {}
    for name, fn, nbytes, stream in (("h2d", lambda st: st["dev_in"].copy_(st["host_in"], non_blocking=True), h2d, up),
                                     ("d2h", lambda st: st["host_out"].copy_(st["dev_out"], non_blocking=True), d2h,
                                      down)):
        barrier()
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        with torch.cuda.stream(stream):
            c0.record(stream)
            for r in range(reps):
                fn(sets[r % 2])
            c1.record(stream)
        torch.cuda.synchronize()
        cms = c0.elapsed_time(c1) / reps
        if world > 1:
            import torch.distributed as dist
            t = torch.tensor([cms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            cms = t.item()
        copies[name] = {"bytes": nbytes, "ms": round(cms, 4), "gbs_per_rank": round(nbytes / (cms / 1e3) / 1e9, 2),
                        "gbs_all_ranks": round(world * nbytes / (cms / 1e3) / 1e9, 1)}
    barrier()
    return {"value": round(step_bytes * args.steps * world / (ms / 1e3) / 1e9, 1), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms / args.steps, 4),
            "host_copies": copies, "numa_node": numa["node"],
            "path": "pinned host -> HBM copy, 24 C-ABI decode launches (CUDA graph), HBM -> pinned host copy; "
                    "uploads/downloads of neighbouring steps overlap compute on two copy streams"}


def run_chunk_bench(args, world, barrier, peaks, seed):
    """Config-2 shard on each GPU: B=8, T=32768, bf16 q/k/v, fp32 state; the
    time is the max over ranks."""
    import torch

    from orionsbelt_b200 import _lib, ops, synth

    c = CFG2_SHARD
    d = synth.device_gdn(c["B"], c["T"], c["Hk"], c["Hv"], c["dk"], c["dv"], g_scale=0.1, seed=seed + 77,
                         in_dtype=torch.bfloat16)
    o = torch.empty_like(d["v"])
    S = d["S0"].clone()
    a = ops.chunk_args(d["q"], d["k"], d["v"], d["g"], d["beta"], S, o, scale=1.0)
    L = _lib.lib()
    stream = torch.cuda.current_stream()
    flush = L2Flush()
    for _ in range(1):
        _lib.check(L.kai_run_gdn_chunk_delta_rule_sm100a(a, stream.cuda_stream))
    barrier()
    reps = max(1, min(args.steps, 3))
    tot = 0.0
    for _ in range(reps):
        flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        _lib.check(L.kai_run_gdn_chunk_delta_rule_sm100a(a, stream.cuda_stream))
        e1.record(stream)
        torch.cuda.synchronize()
        tot += e0.elapsed_time(e1)
    ms = tot / reps
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    flops = metrics.chunk_flops(c["B"], c["T"], c["Hv"], c["dk"], 64) * world
    nbytes = metrics.chunk_bytes(c["B"], c["T"], c["Hk"], c["Hv"], c["dk"], c["dv"], e_in=2, e_out=2, e_state=4) * world
    tok = c["B"] * c["T"] * world / (ms / 1e3)
    return {"workload": "config 2 shard per GPU: B=8, T=32768, 16/32 heads, 128x128, bf16 q/k/v/o, fp32 state "
                        "(aggregate tokens/s and TF/s over all GPUs; fractions per GPU)",
            "kernel": "chunk_ws_kernel<bf16> (warp-specialised: TMA loads, tcgen05 MMAs, fp32 state in TMEM)",
            "tokens_per_s": round(tok, 1), "ms": round(ms, 3),
            "tflops": round(flops / (ms / 1e3) / 1e12, 2), "gbs": round(nbytes / (ms / 1e3) / 1e9, 1),
            "tensor_frac_of_bf16_peak": round(flops / world / (ms / 1e3) / 1e12 / peaks["bf16_tflops"], 4),
            "hbm_frac": round(nbytes / world / (ms / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
            "l2": "256 MB buffer written, then a 256 MB buffer read, before each timed call"}


def run_strong(args, world, rank, barrier, peaks):
    """Strong scaling: the fixed global problem split over the ranks with
    shard.batch_slice, no exchange (max over ranks of each rank's device time).
      decode: config 1's B = 64 global sequences, 24 layers (64 / N per rank);
      chunk:  config 2's B = 8 sequences x 32 value heads (8 / N per rank).
    At N = 8 each rank holds one config-2 sequence (32 (b, h) units): the
    sequential state pass per unit is what bounds that point."""
    import torch
    import torch.distributed as dist

    from orionsbelt_b200 import _lib, ops, shard, synth

    L = _lib.lib()
    out = {}

    def tmax(ms):
        if world > 1:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = t.item()
        return ms

    c = CFG1
    b0, b1 = shard.batch_slice(c["B"], world, rank)
    Bl = b1 - b0
    layers = []
    for layer in range(c["layers"]):
        d = synth.device_gdn(Bl, 1, c["Hk"], c["Hv"], c["dk"], c["dv"], g_scale=0.1, seed=500 + layer,
                             in_dtype=torch.bfloat16, state_std=0.02)
        o = torch.empty((Bl, c["Hv"], c["dv"]), dtype=torch.bfloat16, device="cuda")
        layers.append((d, o, ops.decode_args(d["S0"], d["q"][:, 0].contiguous(), d["k"][:, 0].contiguous(),
                                             d["v"][:, 0].contiguous(), d["g"][:, 0].contiguous(),
                                             d["beta"][:, 0].contiguous(), o, scale=1.0)))
    launch = L.kai_run_gdn_delta_rule_decode_sm100a

    def step():
        sp = torch.cuda.current_stream().cuda_stream
        for _, _, a in layers:
            _lib.check(launch(a, sp))

    step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for _ in range(args.warmup):
        g.replay()
    barrier()
    K = args.steps
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = tmax(e0.elapsed_time(e1) / K)
    barrier()
    del g
    gbytes = metrics.decode_bytes(c["B"], c["Hk"], c["Hv"], c["dk"], c["dv"]) * c["layers"]
    out["decode_cfg1"] = {"global_batch": c["B"], "batch_per_rank": Bl, "ms_per_step": round(ms, 4),
                          "gbs": round(gbytes / (ms / 1e3) / 1e9, 1),
                          "gbs_per_gpu": round(gbytes / world / (ms / 1e3) / 1e9, 1)}
    del layers
    torch.cuda.empty_cache()
    if not args.no_chunk:
        cc = CFG2_SHARD
        b0, b1 = shard.batch_slice(cc["B"], world, rank)
        Bl = b1 - b0
        d = synth.device_gdn(Bl, cc["T"], cc["Hk"], cc["Hv"], cc["dk"], cc["dv"], g_scale=0.1, seed=600 + rank,
                             in_dtype=torch.bfloat16)
        o = torch.empty_like(d["v"])
        S = d["S0"].clone()
        a = ops.chunk_args(d["q"], d["k"], d["v"], d["g"], d["beta"], S, o, scale=1.0)
        sp = torch.cuda.current_stream().cuda_stream
        _lib.check(L.kai_run_gdn_chunk_delta_rule_sm100a(a, sp))
        flush = L2Flush()
        barrier()
        flush()
        e0.record()
        _lib.check(L.kai_run_gdn_chunk_delta_rule_sm100a(a, sp))
        e1.record()
        torch.cuda.synchronize()
        ms = tmax(e0.elapsed_time(e1))
        barrier()
        flops = metrics.chunk_flops(cc["B"], cc["T"], cc["Hv"], cc["dk"], 64)
        out["chunk_cfg2"] = {"global_batch": cc["B"], "batch_per_rank": Bl, "units_per_rank": Bl * cc["Hv"],
                             "ms": round(ms, 3), "tokens_per_s": round(cc["B"] * cc["T"] / (ms / 1e3), 1),
                             "tflops": round(flops / (ms / 1e3) / 1e12, 2),
                             "tensor_frac_per_gpu": round(flops / world / (ms / 1e3) / 1e12 / peaks["bf16_tflops"], 4)}
        del d, o, S
        torch.cuda.empty_cache()
    return out


CFG4 = dict(hidden=2560, vocab=151936, inter=9216, is_gdn=[1, 1, 1, 0] * 8, gdn_heads_k=16, gdn_heads_v=32,
            gdn_head_dim=128, attn_heads=16, attn_kv_heads=4, attn_head_dim=256, rope_dims=64, rope_theta=1e7,
            rms_eps=1e-6, weight_std=0.02)


def run_model(args, world, rank, barrier, peaks, ctx=32768, steps=256):
    """the Qwen3.5-4B-style hybrid (kai_gdn_model_*),
    tensor-parallel over all ranks (NCCL all-reduce after every output
    projection, all-gather of the argmax).  At batch 1 and at batch 16: a
    `ctx`-token prompt of uniform random token ids per sequence through
    kai_gdn_model_prefill (timed), then 256 greedy decode steps from the
    state it left (timed).  Device time with CUDA events, max over ranks; the
    generated tokens are read back to the host once, after the last step."""
    import torch
    import torch.distributed as dist

    from orionsbelt_b200 import ops

    out = {}

    def fresh_id():  # an NCCL unique id serves one communicator: one per engine
        if world == 1:
            return None
        box = [ops.ModelEngine.nccl_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        return box[0]

    geom = dict(CFG4, max_ctx=ctx + steps + 8)
    H, L = geom["hidden"], len(geom["is_gdn"])
    # int8 weight bytes one token streams on each GPU (all layers + LM head), for the roofline
    d, hk, hv, D, hq, hkv_g, I, V = 128, 16, 32, 256, 16, 4, 9216, 151936
    gdn_in = H * ((2 * hk + 2 * hv) * d + 2 * hv)
    gdn_w = gdn_in + hv * d * H
    att_w = H * (hq * 2 * D + 2 * hkv_g * D) + hq * D * H
    ffn_w = 3 * H * I
    tok_bytes = (24 * (gdn_w + ffn_w) + 8 * (att_w + ffn_w) + H * V) / world
    stream = torch.cuda.Stream()
    for B in (1, 16):
        eng = ops.ModelEngine(geom, B, seed=42, tp_rank=rank, tp_size=world, nccl_id=fresh_id())
        prompt = np.random.default_rng(9 + B).integers(0, geom["vocab"], (B, ctx)).astype(np.int32)
        with torch.cuda.stream(stream):
            eng.prefill(prompt[:, :512], 0, stream)  # the prompt workspace and the kernels' first launches
            eng.reset()
            barrier()
            p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            p0.record(stream)
            eng.prefill(prompt, 0, stream)
            p1.record(stream)
            stream.synchronize()
        pms = p0.elapsed_time(p1)
        if world > 1:
            t = torch.tensor([pms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            pms = t.item()
        out[f"prefill_b{B}"] = {"tokens": B * ctx, "s": round(pms / 1e3, 4),
                                "tokens_per_s": round(B * ctx / (pms / 1e3), 1),
                                "first_tokens": [int(x) for x in eng.tokens()[:4]]}
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            for w in range(3):  # eager step, graph capture, one replay
                eng.step(ctx + w, stream)
            stream.synchronize()
            barrier()
            e0.record(stream)
            for i in range(steps):
                eng.step(ctx + 3 + i, stream)
            e1.record(stream)
            stream.synchronize()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = t.item()
        toks = eng.tokens()
        per = ms / steps
        out[f"b{B}"] = {"batch": B, "steps": steps, "ms_per_step": round(per, 4),
                        "tokens_per_s": round(B * steps / (ms / 1e3), 1),
                        "weight_gbs_per_gpu": round(tok_bytes / (per / 1e3) / 1e9, 1),
                        "weight_hbm_frac": round(tok_bytes / (per / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
                        "last_tokens": [int(x) for x in toks[:4]]}
        eng.close()
        del eng
        torch.cuda.empty_cache()
        barrier()
    out.update({"workload": f"config 4: Qwen3.5-4B-style hybrid (hidden 2560, 24 GDN + 8 gated-GQA layers, FFN "
                            f"9216, vocab 151936, int8 weights, bf16 KV cache): per sequence a {ctx}-token prompt "
                            f"of uniform random ids (prefill), then {steps} greedy decode steps, at batch 1 and 16; "
                            f"tensor-parallel x{world} over NCCL",
                "kernels": "decode: gemv_int8_kernel / int8_packed_kernel, decode_step_kernel, attn_tc_kernel, model "
                           "elementwise kernels, per-segment CUDA graphs; prefill: int8_gemm_kernel (row-tiled int8 "
                           "tcgen05 GEMM over the packed weights), chunk_prep_kernel + chunk_rec_kernel (fp32 chunk "
                           "scan on tcgen05), attn_prefill_kernel",
                "weight_bytes_per_token_per_gpu": int(tok_bytes)})
    return out


class L2Flush:
    """Write a buffer larger than L2 (126 MB), then read a second one: the
    read evicts the written (dirty) lines, so their write-back to HBM happens
    here and not inside the next timed call, which still finds L2 cold."""

    def __init__(self):
        import torch

        self.w = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
        self.r = torch.zeros(64 * 1024 * 1024, dtype=torch.float32, device="cuda")

    def __call__(self):
        self.w.zero_()
        self.r.sum()


def _time(fn, reps: int, flush=None) -> float:
    """Average milliseconds of fn() over `reps` launches, CUDA events on the
    current stream, optionally writing a buffer larger than L2 before each.
    A short GPU spin (torch.cuda._sleep, bounded) is queued before the start
    event, so the host-side work of the call (argument checks, the ctypes
    call, the launch) overlaps it and the interval is the GPU time of the
    call's own launches."""
    import torch

    stream = torch.cuda.current_stream()
    fn()
    torch.cuda.synchronize()
    tot = 0.0
    for _ in range(reps):
        if flush is not None:
            flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(1_000_000)  # ~0.5 ms at 1.9 GHz
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize()
        tot += e0.elapsed_time(e1)
    return tot / reps


def run_rows(args, peaks) -> dict:
    """One measurement per hot-path row of the scope table, each on its
    configuration's shape, with the HBM (or tensor) roofline fraction."""
    import torch

    from orionsbelt_b200 import ops, synth

    hbm = peaks["hbm_gbs"]
    flush = L2Flush()
    reps = 5
    out = {}

    def bw_row(name, workload, nbytes, ms, kernel):
        out[name] = {"workload": workload, "kernel": kernel, "ms": round(ms, 4),
                     "gbs": round(nbytes / (ms / 1e3) / 1e9, 1),
                     "hbm_frac": round(nbytes / (ms / 1e3) / 1e9 / hbm, 4), "bytes": nbytes}

    # a1: decay cumsum at config 2 (B=8 x T=32768 x 32 log-decays) and the
    # prefix product at config 0 ([2048][32]) and at the e2e's key channels
    g = -torch.nn.functional.softplus(synth.device_normal((8, 32768, 32), 11, 1)) * 0.1
    gc = torch.empty_like(g)
    ms = _time(lambda: ops.cumsum(g, gc), reps, flush)
    bw_row("a1_cumsum_cfg2", "log-decay cumsum, 8 x 32768 x 32 fp32", 2 * g.numel() * 4, ms, "scan_*_kernel<CUMSUM>")
    a = torch.exp(g[0, :2048].contiguous())
    dcy = torch.empty_like(a)
    ms = _time(lambda: ops.cumdecay(a, dcy), reps, flush)
    bw_row("a1_cumdecay_cfg0", "prefix product, 2048 x 32 fp32 (launch-bound size)", 2 * a.numel() * 4, ms,
           "scan_final_kernel<CUMPROD>")
    a2 = torch.rand((4096, 4096), device="cuda") * 0.2 + 0.9
    d2 = torch.empty_like(a2)
    ms = _time(lambda: ops.cumdecay(a2, d2), reps, flush)
    bw_row("a1_cumdecay_4096x4096", "prefix product, 4096 x 4096 fp32", 2 * a2.numel() * 4, ms,
           "scan_*_kernel<CUMPROD>")
    del g, gc, a, dcy, a2, d2
    # a2: conv at config 0 (fp32, T=2048, 8192 channels) and a config-3 shard (fp16 I/O)
    x, w = synth.device_normal((2048, 8192), 12, 1), synth.device_normal((4, 8192), 12, 2, std=0.5)
    o, hist = torch.empty_like(x), torch.zeros((3, 8192), device="cuda")
    ms = _time(lambda: ops.causal_dwconv1d(x, w, o, hist), reps, flush)
    bw_row("a2_conv_cfg0", "causal dwconv k4, T=2048 x 8192 ch fp32", metrics.conv_bytes(1, 2048, 8192, 4), ms,
           "conv_k4_kernel<f32,4>")
    xh = synth.device_normal((8, 8192, 8192), 12, 3, dtype=torch.float16)
    oh, hh = torch.empty_like(xh), torch.zeros((8, 3, 8192), device="cuda", dtype=torch.float16)
    ms = _time(lambda: ops.causal_dwconv1d(xh, w, oh, hh), reps, flush)
    bw_row("a2_conv_cfg3_shard", "causal dwconv k4, 8 x 8192 x 8192 ch fp16 I/O (config-3 shard)",
           metrics.conv_bytes(8, 8192, 8192, 2), ms, "conv_k4_kernel<f16,8>")
    del x, w, o, hist, xh, oh, hh
    # a3: gated scan over the e2e's value channels (4096) for a 32768-token prefill
    gs = torch.sigmoid(synth.device_normal((32768, 4096), 13, 1))
    xs = synth.device_normal((32768, 4096), 13, 2)
    ss, st = torch.empty_like(xs), torch.zeros(4096, device="cuda")
    ms = _time(lambda: ops.gated_scan(gs, xs, ss, st), reps, flush)
    bw_row("a3_gated_scan", "gated scan, 32768 x 4096 fp32", metrics.gated_scan_bytes(1, 32768, 4096), ms,
           "scan_*_kernel<AFFINE>")
    del gs, xs, ss, st
    # a4: delta-rule GEMV (decode k.S over 32 heads) and matmul (one chunk, 16 heads)
    av, B1 = torch.randn(128, device="cuda"), torch.randn((128, 4096), device="cuda")
    cv = torch.empty(4096, device="cuda")
    ms = _time(lambda: ops.matmul(av[None], B1, cv[None]), reps, flush)
    bw_row("a4_gemv", "GEMV K=128 N=4096 fp32", metrics.matmul_bytes(1, 128, 4096), ms, "gemv_slab_kernel")
    Am, Bm = torch.randn((64, 128), device="cuda"), torch.randn((128, 2048), device="cuda")
    Cm = torch.empty((64, 2048), device="cuda")
    ms = _time(lambda: ops.matmul(Am, Bm, Cm), reps, flush)
    bw_row("a4_matmul", "matmul M=64 K=128 N=2048 fp32 (reference op order)", metrics.matmul_bytes(64, 128, 2048),
           ms, "sgemm_fullk_kernel")
    out["a4_matmul"]["tflops"] = round(2 * 64 * 128 * 2048 / (ms / 1e3) / 1e12, 3)
    del av, B1, cv, Am, Bm, Cm
    # a5: the GDN-1 decode step on one config-1 layer, timed like the f4 row
    # (one launch after the L2 flush) for the comparison; the headline times 24
    d = synth.device_gdn(64, 1, 16, 32, 128, 128, g_scale=0.1, seed=15, in_dtype=torch.bfloat16, state_std=0.02)
    q1, k1, v1, g1, b1 = (d[n][:, 0].contiguous() for n in ("q", "k", "v", "g", "beta"))
    o1 = torch.empty((64, 32, 128), dtype=torch.bfloat16, device="cuda")
    S1 = d["S0"]
    ms = _time(lambda: ops.delta_rule_decode(S1, q1, k1, v1, g1, b1, o1, scale=1.0), reps, flush)
    bw_row("a5_decode_cfg1_layer", "GDN-1 decode step, one config-1 layer, one launch after the L2 flush",
           metrics.decode_bytes(64, 16, 32, 128, 128), ms, "decode_step_kernel<128, f32>")
    del d, q1, k1, v1, g1, b1, o1, S1
    # f4: the GDN-2 decode step (per-channel decay, erase and write gates) on
    # one config-1 layer: B=64, 16 key / 32 value heads, 128x128 fp32 state
    d = synth.device_gdn(64, 1, 16, 32, 128, 128, g_scale=0.1, seed=15, in_dtype=torch.bfloat16, state_std=0.02)
    g2 = -torch.nn.functional.softplus(synth.device_normal((64, 32, 128), 15, 1)) * 0.1
    bg2 = torch.sigmoid(synth.device_normal((64, 32, 128), 15, 2))
    wg2 = torch.sigmoid(synth.device_normal((64, 32, 128), 15, 3))
    o2 = torch.empty((64, 32, 128), dtype=torch.bfloat16, device="cuda")
    q2, k2, v2 = (d[n][:, 0].contiguous() for n in ("q", "k", "v"))
    S2 = d["S0"]
    ms = _time(lambda: ops.gdn2_delta_rule_decode(S2, q2, k2, v2, g2, bg2, wg2, o2, scale=1.0), reps, flush)
    bw_row("f4_gdn2_decode_cfg1", "GDN-2 decode step, one config-1 layer (B=64, 16/32 heads, 128x128 fp32 state, "
           "bf16 q/k/v/o, fp32 per-channel gates)", metrics.gdn2_decode_bytes(64, 16, 32, 128, 128), ms,
           "decode_step_kernel<128, f32, GDN-2>")
    del d, g2, bg2, wg2, o2, q2, k2, v2, S2
    # f2: int8-weight GEMV / small GEMM at the config-4 shapes (hidden 2560,
    # FFN 9216, vocab 151936): the row-major drop-in (kai_run_gdn_matmul_int8)
    # and the packed-weight tensor-core stream (kai_run_gdn_matmul_int8_packed)
    kern_rm = {1: "gemv_int8_kernel (row-major weights, TMA ring)", 16: "matmul_int8_tc_kernel (row-major weights)"}
    for name, (M, K, N), packed in [("f2_int8_gemv_ffn_up", (1, 2560, 9216), False),
                                    ("f2_int8_gemv_ffn_down", (1, 9216, 2560), False),
                                    ("f2_int8_gemm_b16_ffn_up", (16, 2560, 9216), False),
                                    ("f2_int8_packed_b16_ffn_up", (16, 2560, 9216), True),
                                    ("f2_int8_packed_b16_ffn_down", (16, 9216, 2560), True),
                                    ("f2_int8_packed_b16_gate_up", (16, 2560, 18432), True),
                                    ("f2_int8_packed_lm_head_b1", (1, 2560, 151936), True),
                                    ("f2_int8_packed_lm_head_b16", (16, 2560, 151936), True)]:
        W = synth.device_normal((K, N), 16, 1, std=0.05)
        q8 = torch.empty((K, N), dtype=torch.int8, device="cuda")
        s8 = torch.empty(N, device="cuda")
        ops.quantize_int8(W, q8, s8)
        del W
        A8 = synth.device_normal((M, K), 16, 2)
        C8 = torch.empty((M, N), device="cuda")
        if packed:
            qp = ops.pack_int8(q8)
            ms = _time(lambda A8=A8, qp=qp, s8=s8, C8=C8: ops.matmul_int8_packed(A8, qp, s8, C8), reps, flush)
            kern = "act_terms_kernel + int8_packed_kernel (kind::i8 tcgen05, stream-K)"
            del qp
        else:
            ms = _time(lambda A8=A8, q8=q8, s8=s8, C8=C8: ops.matmul_int8(A8, q8, s8, C8), reps, flush)
            kern = kern_rm[M]
        bw_row(name, f"int8 weights x fp32 activations, M={M} K={K} N={N} (per-column scales"
               f"{', weights packed once' if packed else ''}), one call after the L2 flush",
               metrics.int8_matmul_bytes(M, K, N), ms, kern)
        del q8, s8, A8, C8
    # f3: GQA attention decode at the config-4 geometry (16 query / 4 kv
    # heads, head_dim 256) over a 32768-token cache: bf16 at batch 1 and 16,
    # int8 (per-head scales) at batch 1
    for name, B, cdt, ctx in [("f3_attn_decode_bf16_b1", 1, torch.bfloat16, 32768),
                              ("f3_attn_decode_bf16_b16", 16, torch.bfloat16, 32768),
                              ("f3_attn_decode_int8_b1", 1, torch.int8, 32768)]:
        H, Hkv, D = 16, 4, 256
        if cdt == torch.int8:
            kc = torch.randint(-128, 128, (B, ctx, Hkv, D), dtype=torch.int8, device="cuda")
            vc = torch.randint(-128, 128, (B, ctx, Hkv, D), dtype=torch.int8, device="cuda")
            ksc = torch.full((B, Hkv), 0.01, device="cuda")
            vsc = torch.full((B, Hkv), 0.01, device="cuda")
        else:
            kc = synth.device_normal((B, ctx, Hkv, D), 17, 1, dtype=cdt)
            vc = synth.device_normal((B, ctx, Hkv, D), 17, 2, dtype=cdt)
            ksc = vsc = None
        qa = synth.device_normal((B, H, D), 17, 3)
        kna, vna = synth.device_normal((B, Hkv, D), 17, 4), synth.device_normal((B, Hkv, D), 17, 5)
        oa = torch.empty((B, H, D), device="cuda")
        ms = _time(lambda: ops.attention_decode(qa, kna, vna, kc, vc, oa, ctx - 1, 0.0625, ksc, vsc), reps, flush)
        bw_row(name, f"GQA decode, B={B}, 16 q / 4 kv heads x 256, {ctx}-token {cdt} KV cache",
               metrics.attn_decode_bytes(B, ctx, H, Hkv, D, kc.element_size()), ms,
               ("attn_tc_kernel" if cdt == torch.bfloat16 else "attn_split_kernel") + " + attn_combine_kernel")
        del kc, vc, qa, kna, vna, oa
    torch.cuda.empty_cache()
    # f1: the reference's end-to-end decode loop at its default (4B) geometry:
    # 32 layers (24 GDN stand-in + 8 simulated attention), SwiGLU FFN, one int8
    # weight set shared by all layers (128 MB); batch 1 and 16, one token per
    # step, replayed as a CUDA graph on a side stream
    import numpy as np
    dims = (2560, 2048, 4096, 8192, 9216, 16, 4, 256, 32)
    rng = np.random.default_rng(18)
    W = {n: (rng.standard_normal(sh, dtype=np.float32) * 0.005) for n, sh in synth.e2e_weight_shapes(dims).items()}
    W["g_beta"] = rng.uniform(0, 1, W["g_beta"].shape).astype(np.float32)
    wbytes = sum(W[n].size for n in W if n not in ("g_conv_w", "g_beta"))  # int8 weights per layer set
    gdn_w = sum(W[n].size for n in ("g_q_proj", "g_k_proj", "g_v_proj", "g_o_proj"))
    att_w = sum(W[n].size for n in ("f_q_proj", "f_k_proj", "f_v_proj", "f_o_proj"))
    ffn_w = sum(W[n].size for n in ("gate_proj", "up_proj", "down_proj"))
    tok_bytes = 24 * gdn_w + 8 * att_w + 32 * ffn_w  # int8 weight bytes streamed per token
    side = torch.cuda.Stream()
    for B in (1, 16):
        eng = ops.E2EEngine(dims, synth.e2e_layer_pattern(32), B, W)
        x = synth.device_normal((B, 2560), 18, 2)
        y = torch.empty_like(x)
        with torch.cuda.stream(side):
            for _ in range(3):
                eng.step(x, y)  # eager, then graph capture, then replay
            side.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            nstep = 10
            e0.record(side)
            for _ in range(nstep):
                eng.step(x, y)
            e1.record(side)
            e1.synchronize()
        ms = e0.elapsed_time(e1) / nstep
        out[f"f1_e2e_decode_b{B}"] = {
            "workload": f"end-to-end decode loop, 4B geometry (32 layers, hidden 2560, FFN 9216), int8 weights "
                        f"({wbytes / 1e6:.0f} MB, shared by all layers as in the reference), batch {B}",
            "kernel": "matmul_int8_stream_kernel + conv / scan / elementwise (one CUDA graph per token)",
            "ms": round(ms, 4), "tokens_per_s": round(B / (ms / 1e3), 1),
            "weight_gbs": round(tok_bytes / (ms / 1e3) / 1e9, 1),
            "note": "weights stay L2-resident across layers (128 MB set)"}
        eng.close()
        del x, y
    del W
    # a6: chunk scan at config 0 (fp32 throughout) and config 3 (fp16 in, fp16 state, strong decay)
    for name, c, dt, sdt, kern in [
            ("a6_chunk_cfg0", dict(B=1, T=2048, g=0.1), torch.float32, torch.float32,
             "chunk_prep_kernel + chunk_rec_kernel (tcgen05, fp32-accurate: three bf16 MMAs per product)"),
            ("a6_chunk_cfg3", dict(B=32, T=8192, g=1.0), torch.float16, torch.float16,
             "chunk_ws_kernel<f16> (warp-specialised, tcgen05)")]:
        d = synth.device_gdn(c["B"], c["T"], 16, 32, 128, 128, g_scale=c["g"], seed=14, in_dtype=dt,
                             state_dtype=sdt)
        oo = torch.empty_like(d["v"])
        S0 = d["S0"]

        def run(d=d, oo=oo, S0=S0):
            ops.chunk_delta_rule(d["q"], d["k"], d["v"], d["g"], d["beta"], S0, oo, scale=1.0)

        ms = _time(run, 2 if c["B"] > 1 else reps, flush)
        fl = metrics.chunk_flops(c["B"], c["T"], 32, 128, 64)
        nb = metrics.chunk_bytes(c["B"], c["T"], 16, 32, 128, 128, e_in=dt.itemsize, e_out=dt.itemsize,
                                 e_state=sdt.itemsize)
        out[name] = {"workload": f"B={c['B']}, T={c['T']}, 16/32 heads, 128x128, in {dt}, state {sdt}",
                     "kernel": kern, "ms": round(ms, 3), "tokens_per_s": round(c["B"] * c["T"] / (ms / 1e3), 1),
                     "tflops": round(fl / (ms / 1e3) / 1e12, 2),
                     "gbs": round(nb / (ms / 1e3) / 1e9, 1)}
        del d, oo, S0
    torch.cuda.empty_cache()
    return out


def gpu_numa_node(device: int) -> dict:
    """NUMA node of a GPU (from its PCI device in sysfs) and that node's CPUs
    (empty when unknown)."""
    import torch
    try:
        bus = torch.cuda.get_device_properties(device).pci_bus_id.lower()
    except (AttributeError, RuntimeError):
        return {"node": None, "cpus": set()}
    parts = bus.split(":")
    if len(parts[0]) == 8:  # 00000000:1b:00.0 -> 0000:1b:00.0
        bus = parts[0][4:] + ":" + ":".join(parts[1:])
    try:
        node = int(Path(f"/sys/bus/pci/devices/{bus}/numa_node").read_text().strip())
    except (OSError, ValueError):
        return {"node": None, "cpus": set()}
    cpus = set()
    if node >= 0:
        try:
            for part in Path(f"/sys/devices/system/node/node{node}/cpulist").read_text().strip().split(","):
                a, _, b = part.partition("-")
                cpus.update(range(int(a), int(b or a) + 1))
        except (OSError, ValueError):
            cpus = set()
    try:
        cpus &= os.sched_getaffinity(0)
    except AttributeError:
        pass
    return {"node": node, "cpus": cpus}


def host_threads() -> int:
    """Host threads this process may run on (its CPU affinity), set explicitly
    for every CPU measurement: a launcher such as torchrun exports
    OMP_NUM_THREADS=1, which must not decide the baseline's thread count."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def host_info(nthreads: int) -> dict:
    model = "unknown"
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                model = ln.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"cpu": model, "threads_used": nthreads, "nproc": os.cpu_count()}


def _cpu_time(fn, min_s: float = 1.0, min_reps: int = 3, max_reps: int = 50) -> dict:
    """p50 / p95 seconds per call after one discarded warm-up call (the
    reference protocol, docs/METRICS.md:393-456, asks for >= 5 timed repeats
    after warm-ups; small calls get more, large ones at least three)."""
    fn()
    ts = []
    t_all = time.perf_counter()
    while len(ts) < max_reps and (len(ts) < min_reps or time.perf_counter() - t_all < min_s):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    ts.sort()
    return {"p50": ts[len(ts) // 2], "p95": ts[min(len(ts) - 1, int(0.95 * len(ts)))], "reps": len(ts)}


def _decode_inputs(r, B, Hk, Hv, dk, dv, state_std=0.02):
    """One config-1 layer's host inputs; q/k/v rounded to bf16 (the GPU arm's
    input type), g and beta fp32."""
    import oracle
    from orionsbelt_b200 import synth

    rb = lambda a: oracle.u16_to_f32(oracle.f32_to_u16(a, "bf16"), "bf16")  # noqa: E731
    S = (r.standard_normal((B, Hv, dk, dv), dtype=np.float32) * state_std) if state_std else None
    q = rb(synth.l2norm(r.standard_normal((B, Hk, dk))))
    k = rb(synth.l2norm(r.standard_normal((B, Hk, dk))))
    v = rb(r.standard_normal((B, Hv, dv)).astype(np.float32))
    beta = (1 / (1 + np.exp(-r.standard_normal((B, Hv))))).astype(np.float32)
    g = (-synth.softplus(r.standard_normal((B, Hv))) * 0.1).astype(np.float32)
    return S, q, k, v, g, beta


def cpu_decode_sample(seconds: float = 5.0, nthreads: int = 0) -> dict:
    """Oracle port of ref_delta_rule (gpu/gdn_gpu_validate.c:100-118), OpenMP over
    (batch, head) on `nthreads` host threads, on one config-1 layer at B=64
    (bf16-rounded q/k/v, the state updated in place), repeated for ~`seconds`.
    Bytes are counted as for the GPU arm."""
    import oracle

    orc, _ = oracle.require()
    nthreads = nthreads or host_threads()
    orc.set_threads(nthreads)
    c = CFG1
    r = np.random.default_rng(5)
    S, q, k, v, g, beta = _decode_inputs(r, c["B"], c["Hk"], c["Hv"], c["dk"], c["dv"])
    layer_bytes = metrics.decode_bytes(c["B"], c["Hk"], c["Hv"], c["dk"], c["dv"], e_state=4, e_in=2, e_out=2)
    orc.delta_rule_decode(S, q, k, v, g, beta, nthreads=nthreads, copy=False)
    n, t_start = 0, time.perf_counter()
    while True:
        orc.delta_rule_decode(S, q, k, v, g, beta, nthreads=nthreads, copy=False)
        n += 1
        el = time.perf_counter() - t_start
        if el >= seconds:
            break
    return {"value": round(layer_bytes * n / el / 1e9, 3), "unit": "GB/s", "cores": nthreads, "kind": "port",
            "sample": f"{n} x one config-1 layer (B=64, 32 heads, 128x128 fp32 state updated in place, bf16-rounded "
                      f"q/k/v), {el:.1f} s, OpenMP over (batch, head) on {nthreads} threads; oracle restatement of "
                      f"gpu/gdn_gpu_validate.c:100-118 (the reference's C decode step is in an OpenCL host file "
                      f"that does not build here)", "host": host_info(nthreads)}


def cpu_rows(nthreads: int) -> dict:
    """CPU baseline of every per-row measurement, on this host's cores: the
    reference's own C (oracle/_ref, compiled from its sources; kind
    "reference") where the reference has code for the row, else the oracle
    restatement (kind "port").  kai_run_* kernels are single-threaded by
    design; gdn_sve.c's gdn_* twins and the oracle's loops run OpenMP on
    `nthreads` threads.  Chunk rows: the reference has no chunked
    implementation, so the CPU figure is the token loop (the recurrence the
    chunked form restates), timed on a sample of (batch, head) pairs and
    tokens and extrapolated to the configuration's tokens/s."""
    import oracle
    from orionsbelt_b200 import synth

    orc, ref = oracle.require()
    orc.set_threads(nthreads)
    r = np.random.default_rng(31)
    f32 = lambda *sh: r.standard_normal(sh, dtype=np.float32)  # noqa: E731
    out = {}

    def bw(name, nbytes, fn, kind, cores, sample):
        t = _cpu_time(fn)
        out[name] = {"value": round(nbytes / t["p50"] / 1e9, 4), "unit": "GB/s", "cores": cores, "kind": kind,
                     "ms_p50": round(t["p50"] * 1e3, 3), "ms_p95": round(t["p95"] * 1e3, 3), "reps": t["reps"],
                     "sample": sample}

    def have(lib):
        return lib is not None

    P = lambda a: a.ctypes.data_as(oracle.C.POINTER(oracle.C.c_float))  # noqa: E731
    sz = oracle.C.c_size_t

    # a1: log-decay cumsum (the reference has the prefix product only: port)
    g = (-synth.softplus(f32(8, 32768, 32)) * 0.1).astype(np.float32)
    bw("a1_cumsum_cfg2", 2 * g.size * 4, lambda: [orc.cumsum(g[b]) for b in range(8)], "port", 1,
       "full size, 8 x 32768 x 32, oracle cumsum (single thread)")
    a0 = np.exp(g[0, :2048]).astype(np.float32)
    a4k = (r.uniform(0.9, 1.1, (4096, 4096))).astype(np.float32)
    if have(ref):
        o0 = np.empty_like(a0)
        bw("a1_cumdecay_cfg0", 2 * a0.size * 4,
           lambda: ref.lib.kai_run_gdn_cumdecay_f32_sve(P(a0), P(o0), sz(2048), sz(32)), "reference", 1,
           "full size, 2048 x 32, kai_run_gdn_cumdecay_f32_sve (single-threaded by design)")
        bw("a1_cumdecay_4096x4096", 2 * a4k.size * 4, lambda: ref.cumdecay(a4k), "reference", nthreads,
           f"full size, gdn_cumdecay_f32 (gdn_sve.c, OpenMP, {nthreads} threads)")
    # a2: conv, config 0 (reference, OpenMP) and the config-3 fp16 shard (port, sampled rows)
    x0, w0, h0 = f32(2048, 8192), (f32(4, 8192) * 0.5).astype(np.float32), np.zeros((3, 8192), np.float32)
    if have(ref):
        bw("a2_conv_cfg0", metrics.conv_bytes(1, 2048, 8192, 4), lambda: ref.conv(x0, w0, h0), "reference",
           nthreads, f"full size, 2048 x 8192 fp32, gdn_causal_dwconv1d_f32 (gdn_sve.c, OpenMP, {nthreads} threads)")
    xh = oracle.f32_to_u16(f32(1024, 8192), "f16")
    hh = np.zeros((3, 8192), np.uint16)
    bw("a2_conv_cfg3_shard", metrics.conv_bytes(1, 1024, 8192, 2), lambda: orc.conv_narrow(xh, w0, hh, "f16"),
       "port", 1, "1024 of 8 x 8192 rows x 8192 channels, fp16 I/O, oracle conv (the reference's conv is fp32 "
       "only), GB/s of the sample")
    # a3: gated scan (reference, OpenMP), 4096 of the 32768 rows
    gs = r.uniform(0.5, 0.99, (4096, 4096)).astype(np.float32)
    xs = f32(4096, 4096)
    st = np.zeros(4096, np.float32)
    if have(ref):
        bw("a3_gated_scan", metrics.gated_scan_bytes(1, 4096, 4096), lambda: ref.gated_scan(gs, xs, st), "reference",
           nthreads, f"4096 of the 32768 rows x 4096 channels, gdn_gated_scan_f32 (gdn_sve.c, OpenMP, {nthreads} "
           f"threads), GB/s of the sample")
        # a4: GEMV (kai, single-threaded) and the delta-rule matmul
        av, B1 = f32(128), f32(128, 4096)
        bw("a4_gemv", metrics.matmul_bytes(1, 128, 4096), lambda: ref.gemv(av, B1), "reference", 1,
           "full size, K=128 N=4096, kai_run_gdn_gemv_f32_f32_f32_1x4_neon (scalar branch, single thread)")
        Am, Bm = f32(64, 128), f32(128, 2048)
        bw("a4_matmul", metrics.matmul_bytes(64, 128, 2048), lambda: ref.matmul(Am, Bm), "reference", 1,
           "full size, M=64 K=128 N=2048, gdn_delta_rule_matmul (scalar path, single thread)")
    # a5 / f4: one config-1 layer, port (OpenMP over (batch, head)), state in place
    S, q, k, v, gd, beta = _decode_inputs(r, 64, 16, 32, 128, 128)
    bw("a5_decode_cfg1_layer", metrics.decode_bytes(64, 16, 32, 128, 128),
       lambda: orc.delta_rule_decode(S, q, k, v, gd, beta, nthreads=nthreads, copy=False), "port", nthreads,
       f"full config-1 layer (B=64), oracle ref_delta_rule restatement, OpenMP over (batch, head) on {nthreads} "
       f"threads, state updated in place")
    g2 = (-synth.softplus(f32(64, 32, 128)) * 0.1).astype(np.float32)
    bg2, wg2 = r.uniform(0, 1, (64, 32, 128)).astype(np.float32), r.uniform(0, 1, (64, 32, 128)).astype(np.float32)
    bw("f4_gdn2_decode_cfg1", metrics.gdn2_decode_bytes(64, 16, 32, 128, 128),
       lambda: orc.gdn2_decode(S, q, k, v, g2, bg2, wg2, nthreads=nthreads), "port", nthreads,
       f"full config-1 layer (B=64), oracle restatement of gdn2_recurrent (bench/gdn2_reference.py:58-145), "
       f"OpenMP on {nthreads} threads")
    del S
    # f2: int8 weights, the reference's own gemv_int8_neon / gemm_int8_neon (scalar branch)
    if oracle.ref_int8 is not None:
        # (the packed rows compute the same product; the reference has one weight layout)
        for names, (M, K, N), Ns in [(("f2_int8_gemv_ffn_up",), (1, 2560, 9216), 9216),
                                     (("f2_int8_gemv_ffn_down",), (1, 9216, 2560), 2560),
                                     (("f2_int8_gemm_b16_ffn_up", "f2_int8_packed_b16_ffn_up"), (16, 2560, 9216), 9216),
                                     (("f2_int8_packed_b16_ffn_down",), (16, 9216, 2560), 2560),
                                     (("f2_int8_packed_b16_gate_up",), (16, 2560, 18432), 18432),
                                     (("f2_int8_packed_lm_head_b1",), (1, 2560, 151936), 151936),
                                     (("f2_int8_packed_lm_head_b16",), (16, 2560, 151936), 151936)]:
            W = (f32(K, Ns) * 0.05).astype(np.float32)
            q8, s8 = oracle.ref_int8.quantize_int8(W)
            A8 = f32(M, K)
            what = "full size" if Ns == N else f"{Ns} of the {N} columns, GB/s of the sample"
            for name in names:
                bw(name, metrics.int8_matmul_bytes(M, K, Ns), lambda A8=A8, q8=q8, s8=s8: oracle.ref_int8.matmul_int8(
                    A8, q8, s8), "reference", 1,
                   f"{what}, M={M} K={K} N={N}, the reference's {'gemv' if M == 1 else 'gemm'}_int8_neon "
                   f"(gdn_e2e_decode.c, scalar branch, single thread)")
    # f3: attention decode over a 32768-token cache; bf16 cache: oracle (the
    # reference's attention has fp32 / int8 caches only); int8: the reference's own
    H, Hkv, D, ctx = 16, 4, 256, 32768
    for name, Bs, Bfull in [("f3_attn_decode_bf16_b1", 1, 1), ("f3_attn_decode_bf16_b16", 2, 16)]:
        qa, kn, vn = f32(Bs, H, D), f32(Bs, Hkv, D), f32(Bs, Hkv, D)
        kc = oracle.f32_to_u16(f32(Bs, ctx, Hkv, D), "bf16")
        vc = oracle.f32_to_u16(f32(Bs, ctx, Hkv, D), "bf16")
        bw(name, metrics.attn_decode_bytes(Bs, ctx, H, Hkv, D, 2),
           lambda qa=qa, kn=kn, vn=vn, kc=kc, vc=vc: orc.attn_decode(qa, kn, vn, kc, vc, ctx - 1, 0.0625,
                                                                   nthreads=nthreads), "port", nthreads,
           f"B={Bs} of {Bfull}, 32768-token bf16 cache, oracle attention decode (OpenMP on {nthreads} threads), "
           f"GB/s of the sample")
        del kc, vc
    qa, kn, vn = f32(1, H, D), f32(1, Hkv, D), f32(1, Hkv, D)
    kc8 = r.integers(-128, 128, (1, ctx, Hkv, D)).astype(np.int8)
    vc8 = r.integers(-128, 128, (1, ctx, Hkv, D)).astype(np.int8)
    sc = np.full((1, Hkv), 0.01, np.float32)
    bw("f3_attn_decode_int8_b1", metrics.attn_decode_bytes(1, ctx, H, Hkv, D, 1),
       lambda: orc.attn_decode(qa, kn, vn, kc8, vc8, ctx - 1, 0.0625, sc, sc, nthreads=nthreads), "port", nthreads,
       f"full size, B=1, 32768-token int8 cache, oracle restatement of full_attn_real_forward_int8kv "
       f"(gdn_e2e_decode.c:1652-1830, bit-identical to it), OpenMP on {nthreads} threads")
    # chunk scans: the token loop on sampled (batch, head) pairs and tokens
    def chunk_row(name, B, T, g_scale, T_sample, pairs, kind_in):
        d = synth.host_gdn(1, T_sample, pairs, pairs, 128, 128, g_scale=g_scale, seed=3)
        if kind_in != "f32":
            for key in ("q", "k", "v"):
                d[key] = oracle.u16_to_f32(oracle.f32_to_u16(d[key], kind_in), kind_in)
        t = _cpu_time(lambda: orc.delta_rule_seq(d["S0"], d["q"], d["k"], d["v"], d["g"], d["beta"],
                                                 nthreads=nthreads), min_s=1.0, min_reps=2)
        pair_tok = pairs * T_sample / t["p50"]
        out[name] = {"value": round(pair_tok / 32, 1), "unit": "tokens/s", "cores": nthreads, "kind": "port",
                     "ms_p50": round(t["p50"] * 1e3, 2), "reps": t["reps"],
                     "sample": f"token loop (oracle restatement of gpu/gdn_gpu_validate.c:100-118; the reference "
                               f"has no chunked implementation) over {pairs} (batch, head) pairs x {T_sample} "
                               f"tokens, OpenMP over pairs on {nthreads} threads; tokens/s of the B={B}, T={T}, "
                               f"32-head configuration extrapolated as pair-tokens/s / 32"}

    chunk_row("a6_chunk_cfg0", 1, 2048, 0.1, 512, 32, "f32")
    chunk_row("chunk_cfg2", 8, 32768, 0.1, 1024, max(nthreads, 8), "bf16")
    chunk_row("a6_chunk_cfg3", 32, 8192, 1.0, 1024, max(nthreads, 8), "f16")
    # f1: the end-to-end loop, oracle restatement at the 4B geometry, one token
    dims = (2560, 2048, 4096, 8192, 9216, 16, 4, 256, 32)
    W = {n: (r.standard_normal(sh, dtype=np.float32) * 0.005) for n, sh in synth.e2e_weight_shapes(dims).items()}
    W["g_beta"] = r.uniform(0, 1, W["g_beta"].shape).astype(np.float32)
    pat = synth.e2e_layer_pattern(32)
    h1 = (f32(1, 1, 2560) * 0.1).astype(np.float32)
    h2 = (f32(2, 1, 2560) * 0.1).astype(np.float32)
    t0 = time.perf_counter()
    orc.e2e_decode(dims, pat, W, h1, nthreads=nthreads)
    t1 = time.perf_counter()
    orc.e2e_decode(dims, pat, W, h2, nthreads=nthreads)
    t2 = time.perf_counter()
    per_tok = max((t2 - t1) - (t1 - t0), 1e-9)
    for name in ("f1_e2e_decode_b1", "f1_e2e_decode_b16"):
        out[name] = {"value": round(1.0 / per_tok, 3), "unit": "tokens/s", "cores": nthreads, "kind": "port",
                     "ms_per_token": round(per_tok * 1e3, 2),
                     "sample": f"decode tokens of one sequence, 4B geometry, int8 weights, oracle restatement of the "
                               f"reference's loop (gdn_e2e_decode.c:2775-2796; its int8 GEMVs split over {nthreads} "
                               f"threads by columns); time per token = (2-token call - 1-token call), so the weight "
                               f"quantization each call repeats is excluded; sequences run one after another, so "
                               f"batch 16 has the same tokens/s"}
    return out


# ---------------------------------------------------------------- reference

def run_reference(args):
    """The reference path's CPU implementation of the headline step: the
    oracle port of ref_delta_rule (the reference's C decode step lives in an
    OpenCL host file that does not build here), on every host thread this
    process may use (set explicitly, whatever OMP_NUM_THREADS a launcher
    exported), over the same workload as the GPU arm: one step = the decode
    step of all 24 config-1 layers at B = 64, bf16-rounded q/k/v, each layer's
    fp32 state updated in place; bytes counted as for the GPU arm."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle

    orc, _ = oracle.require()
    nthreads = host_threads()
    orc.set_threads(nthreads)
    c = CFG1
    r = np.random.default_rng(5)
    base = _decode_inputs(r, c["B"], c["Hk"], c["Hv"], c["dk"], c["dv"])
    layers = []
    for li in range(c["layers"]):
        S = base[0] * np.float32(1.0 + 0.001 * li)  # each layer its own 268 MB state
        layers.append((S,) + _decode_inputs(r, c["B"], c["Hk"], c["Hv"], c["dk"], c["dv"], state_std=0)[1:])
    layer_bytes = metrics.decode_bytes(c["B"], c["Hk"], c["Hv"], c["dk"], c["dv"], e_state=4, e_in=2, e_out=2)
    step_bytes = layer_bytes * c["layers"]

    def step():
        for S, q, k, v, g, beta in layers:
            orc.delta_rule_decode(S, q, k, v, g, beta, nthreads=nthreads, copy=False)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    value = step_bytes * args.steps / el / 1e9
    sample = (f"each step = the full config-1 decode step (24 layers, B=64, 32 value heads, 128x128 fp32 state "
              f"updated in place, bf16-rounded q/k/v) on {nthreads} host threads (OpenMP over (batch, head)); "
              f"oracle port of the reference's ref_delta_rule (gpu/gdn_gpu_validate.c:100-118; that file needs "
              f"OpenCL headers and does not build here)")
    line = {"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config 1: recurrent decode step over 24 GDN layers, batch 64, 32 value / 16 key "
                                   "heads, 128x128 fp32 state, bf16 q/k/v (CPU)", "global_batch": c["B"],
                       "layers": c["layers"], "parallelism": f"OpenMP x{nthreads} over (batch, head)",
                       "bytes_per_step": step_bytes},
            "impl": "reference",
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": nthreads, "kind": "port",
                             "sample": sample, "host": host_info(nthreads)},
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
