"""Algorithmic work of each hot-path operator: the minimal bytes (or FLOPs) one
call must move, used for every GB/s, TFLOP/s and roofline fraction reported.
Bytes are unavoidable traffic, not implementation passes (the reference's own
decode benchmark counts four passes over S, gpu/gdn_gpu_bench.c:673; that is
not used here).
"""
from __future__ import annotations

import re
from pathlib import Path


def cumdecay_bytes(batch, seq, ch, e_out=4):
    """read a + write decay (bench_gdn.c:187 accounting)."""
    return batch * seq * ch * (4 + e_out)


def gated_scan_bytes(batch, seq, ch, e_state=4):
    """read g, x + write s, plus read+write state (bench_kai_gdn.c:331)."""
    return batch * (3 * seq * ch * 4 + 2 * ch * e_state)


def conv_bytes(batch, seq, ch, e_io=4):
    """read in + write out + read w[4][ch] + read/write hist[3][ch]
    (bench_kai_gdn.c:357-360)."""
    return batch * (2 * seq * ch * e_io + 6 * ch * e_io) + 4 * ch * 4


def matmul_bytes(M, K, N):
    """read A, B + write C (bench_kai_gdn.c:377-380 for M=1)."""
    return (M * K + K * N + M * N) * 4


def decode_bytes(B, Hk, Hv, dk, dv, e_state=4, e_in=2, e_out=2):
    """One decode step of one layer: state read + write, q/k per key head, v per
    value head, o per value head, g and beta (fp32) per value head."""
    return (2 * B * Hv * dk * dv * e_state + B * (2 * Hk * dk + Hv * dv) * e_in + B * Hv * dv * e_out
            + 2 * B * Hv * 4)


def gdn2_decode_bytes(B, Hk, Hv, dk, dv, e_state=4, e_in=2, e_out=2):
    """One GDN-2 decode step of one layer: as decode_bytes, with the gates per
    channel (g and b per key channel, w per value channel, fp32)."""
    return (2 * B * Hv * dk * dv * e_state + B * (2 * Hk * dk + Hv * dv) * e_in + B * Hv * dv * e_out
            + B * Hv * (2 * dk + dv) * 4)


def int8_matmul_bytes(M, K, N):
    """int8 weights [K][N] and their fp32 column scales, fp32 A [M][K] and C [M][N]."""
    return K * N + 4 * N + 4 * M * K + 4 * M * N


def attn_decode_bytes(B, ctx, H, Hkv, D, e_cache):
    """One decode step of one attention layer: the K and V caches read once
    (ctx tokens), q and o (fp32), the appended token (read fp32, written)."""
    return 2 * B * ctx * Hkv * D * e_cache + 2 * B * H * D * 4 + 2 * B * Hkv * D * (4 + e_cache)


def chunk_flops(B, T, Hv, d, C=64):
    """Chunkwise scan FLOPs: per (chunk, value head) 6*C*d^2 (W S, Q S, K^T V')
    + 10*C^2*d (K K^T, Q K^T, W, U, P V') + (2/3) C^3 (triangular solve)."""
    n_chunks = -(-T // C)
    return n_chunks * B * Hv * (6 * C * d * d + 10 * C * C * d + (2.0 / 3.0) * C ** 3)


def chunk_bytes(B, T, Hk, Hv, dk, dv, e_in=2, e_out=2, e_state=4):
    """q, k (per key head), v, o per token; g, beta fp32; initial + final state."""
    return (B * T * (2 * Hk * dk + Hv * dv) * e_in + B * T * Hv * 2 * 4 + B * T * Hv * dv * e_out
            + 2 * B * Hv * dk * dv * e_state)


def profiled_traffic(profiles: Path, kernel: str):
    """DRAM bytes per launch of `kernel` recorded from an ncu capture in a
    profiles/*.md summary line of the form
        traffic[<kernel>] = <bytes> bytes/launch
    or None when no capture has been summarised yet."""
    pat = re.compile(r"traffic\[" + re.escape(kernel) + r"\]\s*=\s*([0-9.eE+]+)\s*bytes/launch")
    for f in sorted(Path(profiles).glob("*.md")):
        m = pat.search(f.read_text())
        if m:
            return float(m.group(1))
    return None
