"""GPU parity of the fp32 chunked scan on the tensor cores (chunk_tc32.cu:
chunk_prep_kernel + chunk_rec_kernel, reached through
kai_run_gdn_chunk_delta_rule_sm100a for fp32 q/k/v at dk = 128) against the
oracle's token loop (the reference's ref_delta_rule recurrence).

Bar (written here): relative L2 1e-4, the fp32 bar of the CUDA-core kernel;
every product runs as three bf16 MMAs (about 16 significant bits, fp32
accumulation), measured near 5e-6 on these shapes.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2
from orionsbelt_b200 import ops, synth

pytestmark = pytest.mark.gpu

TOL = 1e-4


def _dev(torch, a, dt=None):
    x = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return x.to(dt) if dt is not None else x


def _run(torch, d, scale, state_dt=None, out_dt=None):
    S = _dev(torch, d["S0"], state_dt)
    o = torch.empty(d["v"].shape, dtype=out_dt or torch.float32, device="cuda")
    ops.chunk_delta_rule(_dev(torch, d["q"]), _dev(torch, d["k"]), _dev(torch, d["v"]), _dev(torch, d["g"]),
                         _dev(torch, d["beta"]), S, o, scale=scale)
    torch.cuda.synchronize()
    return S.float().cpu().numpy(), o.float().cpu().numpy()


@pytest.mark.parametrize("B,T,Hk,Hv,dv,g_scale", [
    (1, 1, 1, 1, 128, 0.3),      # one token
    (1, 64, 1, 1, 128, 0.3),     # exactly one chunk
    (1, 65, 2, 4, 128, 0.3),     # a one-token ragged chunk
    (2, 300, 2, 4, 128, 1.0),    # strong decay, grouped heads
    (1, 200, 4, 4, 128, 0.1),    # one value head per key head
    (1, 130, 1, 2, 64, 0.3),     # dv = 64: two 32-column blocks
    (1, 100, 2, 2, 32, 0.3),     # dv = 32: one block
])
def test_chunk_tc32_vs_token_loop(cuda, orc, B, T, Hk, Hv, dv, g_scale):
    d = synth.host_gdn(B, T, Hk, Hv, 128, dv, g_scale=g_scale, seed=T + dv + Hk, state_std=0.05)
    sc = 1.0 / np.sqrt(128)
    S_want, o_want = orc.delta_rule_seq(d["S0"], d["q"], d["k"], d["v"], d["g"], d["beta"], scale=sc)
    S_got, o_got = _run(cuda, d, sc)
    assert rel_l2(o_got, o_want) < TOL, rel_l2(o_got, o_want)
    assert rel_l2(S_got, S_want) < TOL, rel_l2(S_got, S_want)


@pytest.mark.parametrize("state_kind,out_kind", [("bf16", "f32"), ("f16", "bf16"), ("f32", "f16")])
def test_chunk_tc32_state_and_output_dtypes(cuda, orc, state_kind, out_kind):
    """fp32 inputs with a 16-bit state (loaded and stored at the ends, fp32
    inside) and 16-bit outputs: the bar is the 16-bit rounding of the ends."""
    torch = cuda
    tdt = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}
    d = synth.host_gdn(1, 150, 2, 4, 128, 128, g_scale=0.3, seed=7, state_std=0.05)
    S0 = torch.from_numpy(d["S0"]).to(tdt[state_kind]).float().numpy()
    S_want, o_want = orc.delta_rule_seq(S0, d["q"], d["k"], d["v"], d["g"], d["beta"], scale=0.09)
    S_got, o_got = _run(torch, dict(d, S0=S0), 0.09, state_dt=tdt[state_kind], out_dt=tdt[out_kind])
    tol_s = TOL if state_kind == "f32" else 8e-3
    tol_o = TOL if out_kind == "f32" else 8e-3
    assert rel_l2(o_got, o_want) < tol_o and rel_l2(S_got, S_want) < tol_s


def test_chunk_tc32_segments(cuda, orc):
    """A sequence whose per-chunk images exceed the workspace bound runs in
    segments (B=4, 16/32 heads: 31 chunks per segment, 33 chunks here), the
    state carried through the state buffer; the same bar as one segment."""
    d = synth.host_gdn(4, 33 * 64 - 7, 16, 32, 128, 128, g_scale=0.2, seed=11, state_std=0.05)
    S_want, o_want = orc.delta_rule_seq(d["S0"], d["q"], d["k"], d["v"], d["g"], d["beta"], scale=0.088)
    S_got, o_got = _run(cuda, d, 0.088)
    assert rel_l2(o_got, o_want) < TOL and rel_l2(S_got, S_want) < TOL


def test_chunk_tc32_continuity_and_repeat(cuda, orc):
    """Two calls with the state carried equal one call, and a repeated call is
    bit-identical (no order-dependent reduction)."""
    torch = cuda
    d = synth.host_gdn(1, 256, 2, 4, 128, 128, g_scale=0.2, seed=41, state_std=0.05)
    S_full, o_full = _run(torch, d, 0.125)
    S_again, o_again = _run(torch, d, 0.125)
    assert np.array_equal(S_full, S_again) and np.array_equal(o_full, o_again)
    first = {k: (v[:, :128] if k != "S0" else v) for k, v in d.items()}
    S_mid, o_a = _run(torch, first, 0.125)
    second = {k: (v[:, 128:] if k != "S0" else S_mid) for k, v in d.items()}
    S_end, o_b = _run(torch, second, 0.125)
    assert rel_l2(np.concatenate([o_a, o_b], 1), o_full) < 1e-5 and rel_l2(S_end, S_full) < 1e-5
