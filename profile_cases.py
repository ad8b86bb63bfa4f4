"""Small, self-terminating workloads for ncu captures of one kernel at a time.

    python profile_cases.py decode [--launches 3]
    python profile_cases.py chunk  [--launches 1]
    python profile_cases.py chunk32
    python profile_cases.py conv | cumsum | scan | attn | int8 | int8m16 | lmhead | lmhead16 | ffn16 | model
    python profile_cases.py prefill [--launches 1]
    python profile_cases.py gemm4k
    python profile_cases.py model16

Each case holds a few hundred MB to a few GB on the device (inputs larger
than the 126 MB L2, so DRAM counters mean something), runs a few launches of
its kernel through the C ABI, and exits.  Cases:
  decode  one config-1 layer: B=64, 32 value / 16 key heads, 128x128 fp32
          state (268 MB), bf16 q/k/v/o
  chunk   config-2 numerics on a reduced shard: B=1, T=8192, bf16 in / fp32 state
  chunk32 config 0: B=1, T=2048, 16 key / 32 value heads, fp32 throughout (the
          tensor-core prep and recurrence launches; 67 MB of operand images)
  conv    config-0 Conv1D: T=2048, 8192 channels, fp32 (134 MB)
  cumsum  config-2 decay cumsum: 8 x 32768 x 32 log-decays, fp32
  scan    gated scan, 4096 tokens x 8192 channels, fp32
  attn    GQA attention decode, config-4 heads (16 q / 4 kv x 256), B=4 over a
          32768-token bf16 KV cache (537 MB)
  int8    int8-weight GEMV, M=1, K=2560, N=9216 (23.6 MB of weights)
  int8m16 the same weights, M=16 (the tensor-core path)
  lmhead  int8-weight GEMV over the config-4 LM head, M=1, K=2560, N=151936
          (389 MB of weights)
  lmhead16 the LM head weights packed for streaming, M=16 (the tensor-core
          weight-streaming kernel)
  ffn16   the packed path on the FFN up weights, M=16
  gemm4k  the packed-weight GEMM of a 4096-row prompt block through the
          config-4 GDN input projection (K=2560, N=12352)
  prefill the config-4 engine's prefill of a 32768-token prompt at batch 1
          (one prompt per launch, after a 256-token warm-up prefill)
  model   the config-4 engine (4B geometry, batch 1, synthetic 32k context):
          one greedy decode step per launch
  model16 the same at batch 16
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))

from orionsbelt_b200 import _lib, ops, synth  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["decode", "chunk", "chunk32", "conv", "cumsum", "scan", "attn", "int8", "int8m16", "lmhead",
                                     "lmhead16", "ffn16", "model", "prefill", "gemm4k", "model16"])
    ap.add_argument("--launches", type=int, default=3)
    a = ap.parse_args()
    torch.cuda.set_device(0)
    _lib.lib()
    if a.case == "decode":
        d = synth.device_gdn(64, 1, 16, 32, 128, 128, seed=1, in_dtype=torch.bfloat16, state_std=0.02)
        o = torch.empty((64, 32, 128), dtype=torch.bfloat16, device="cuda")
        args = ops.decode_args(d["S0"], d["q"][:, 0].contiguous(), d["k"][:, 0].contiguous(),
                               d["v"][:, 0].contiguous(), d["g"][:, 0].contiguous(), d["beta"][:, 0].contiguous(),
                               o, scale=1.0)
        fn = lambda: _lib.check(_lib.lib().kai_run_gdn_delta_rule_decode_sm100a(  # noqa: E731
            args, torch.cuda.current_stream().cuda_stream))
    elif a.case == "chunk":
        d = synth.device_gdn(1, 8192, 16, 32, 128, 128, seed=2, in_dtype=torch.bfloat16)
        o = torch.empty_like(d["v"])
        fn = lambda: ops.chunk_delta_rule(d["q"], d["k"], d["v"], d["g"], d["beta"], d["S0"], o)  # noqa: E731
    elif a.case == "chunk32":
        d = synth.device_gdn(1, 2048, 16, 32, 128, 128, seed=2)
        o = torch.empty_like(d["v"])
        fn = lambda: ops.chunk_delta_rule(d["q"], d["k"], d["v"], d["g"], d["beta"], d["S0"], o)  # noqa: E731
    elif a.case == "conv":
        x = synth.device_normal((2048, 8192), 3, 1)
        w = synth.device_normal((4, 8192), 3, 2, std=0.5)
        out = torch.empty_like(x)
        hist = torch.zeros((3, 8192), device="cuda")
        fn = lambda: ops.causal_dwconv1d(x, w, out, hist)  # noqa: E731
    elif a.case == "cumsum":
        g = -torch.nn.functional.softplus(synth.device_normal((8, 32768, 32), 4, 1)) * 0.1
        out = torch.empty_like(g)
        fn = lambda: ops.cumsum(g, out)  # noqa: E731
    elif a.case == "attn":
        kc = synth.device_normal((4, 32768, 4, 256), 6, 1, dtype=torch.bfloat16)
        vc = synth.device_normal((4, 32768, 4, 256), 6, 2, dtype=torch.bfloat16)
        q = synth.device_normal((4, 16, 256), 6, 3)
        kn, vn = synth.device_normal((4, 4, 256), 6, 4), synth.device_normal((4, 4, 256), 6, 5)
        o = torch.empty((4, 16, 256), device="cuda")
        fn = lambda: ops.attention_decode(q, kn, vn, kc, vc, o, 32767, 0.0625)  # noqa: E731
    elif a.case in ("int8", "int8m16"):
        W = synth.device_normal((2560, 9216), 7, 1, std=0.05)
        q8 = torch.empty((2560, 9216), dtype=torch.int8, device="cuda")
        s8 = torch.empty(9216, device="cuda")
        ops.quantize_int8(W, q8, s8)
        M = 16 if a.case == "int8m16" else 1
        A = synth.device_normal((M, 2560), 7, 2)
        Cm = torch.empty((M, 9216), device="cuda")
        fn = lambda: ops.matmul_int8(A, q8, s8, Cm)  # noqa: E731
    elif a.case == "lmhead":
        K, N = 2560, 151936
        W = synth.device_normal((K, N), 8, 1, std=0.02)
        q8 = torch.empty((K, N), dtype=torch.int8, device="cuda")
        s8 = torch.empty(N, device="cuda")
        ops.quantize_int8(W, q8, s8)
        del W
        A = synth.device_normal((1, K), 8, 2)
        Cm = torch.empty((1, N), device="cuda")
        fn = lambda: ops.matmul_int8(A, q8, s8, Cm)  # noqa: E731
    elif a.case in ("lmhead16", "ffn16"):
        K, N = (2560, 151936) if a.case == "lmhead16" else (2560, 9216)
        W = synth.device_normal((K, N), 8, 1, std=0.02)
        q8 = torch.empty((K, N), dtype=torch.int8, device="cuda")
        s8 = torch.empty(N, device="cuda")
        ops.quantize_int8(W, q8, s8)
        del W
        qp = ops.pack_int8(q8)
        del q8
        A = synth.device_normal((16, K), 8, 2)
        Cm = torch.empty((16, N), device="cuda")
        fn = lambda: ops.matmul_int8_packed(A, qp, s8, Cm)  # noqa: E731
    elif a.case == "gemm4k":
        K, N, M = 2560, 12352, 4096
        W = synth.device_normal((K, N), 8, 1, std=0.02)
        q8 = torch.empty((K, N), dtype=torch.int8, device="cuda")
        s8 = torch.empty(N, device="cuda")
        ops.quantize_int8(W, q8, s8)
        del W
        qp = ops.pack_int8(q8)
        del q8
        A = synth.device_normal((M, K), 8, 2)
        Cm = torch.empty((M, N), device="cuda")
        fn = lambda: ops.matmul_int8_packed(A, qp, s8, Cm)  # noqa: E731
    elif a.case == "prefill":
        import numpy as np

        import bench
        T = 32768
        eng = ops.ModelEngine(dict(bench.CFG4, max_ctx=T + 64), 1, seed=42)
        prompt = np.random.default_rng(0).integers(0, bench.CFG4["vocab"], (1, T)).astype(np.int32)
        side = torch.cuda.Stream()
        with torch.cuda.stream(side):
            eng.prefill(prompt[:, :256], 0, side)

        def fn():
            eng.reset()
            with torch.cuda.stream(side):
                eng.prefill(prompt, 0, side)
    elif a.case in ("model", "model16"):
        import numpy as np

        import bench
        nb = 16 if a.case == "model16" else 1
        eng = ops.ModelEngine(dict(bench.CFG4, max_ctx=32768 + 64), nb, seed=42)
        eng.fill(32768, seed=3)
        eng.set_tokens(np.zeros(nb, np.int32))
        side = torch.cuda.Stream()
        step = [0]

        def fn():
            with torch.cuda.stream(side):
                eng.step(32768 + step[0], side)
            step[0] += 1
    else:
        g = torch.sigmoid(synth.device_normal((4096, 8192), 5, 1))
        x = synth.device_normal((4096, 8192), 5, 2)
        s = torch.empty_like(x)
        st = torch.zeros(8192, device="cuda")
        fn = lambda: ops.gated_scan(g, x, s, st)  # noqa: E731
    torch.cuda.synchronize()
    for _ in range(a.launches):
        fn()
    torch.cuda.synchronize()
    print(f"{a.case}: {a.launches} launches ok")


if __name__ == "__main__":
    main()
