"""BASELINE configs 2 and 3 at their full shapes, checked against the oracle.

The chunk scan runs on the whole problem on the GPU (config 2: B=8, T=32768,
16 key / 32 value heads, bf16 q/k/v/o, fp32 state; config 3: B=32, T=8192,
fp16 q/k/v/o, fp16 state storage, g = -softplus(N(0,1))).  The oracle's token
loop (the chunk-free restatement of gpu/gdn_gpu_validate.c:100-118) then runs
a few sampled (batch, value head) pairs over the full sequence on the same
rounded inputs -- about 2 GFLOP per pair at T=32768 -- so the error a long
recurrence accumulates (512 chunks of 16-bit operands) is measured against
the reference arithmetic, not against another GPU kernel.  Narrow state is
widened once on entry and narrowed once on exit (gdn_sve.c:434-441), which
the oracle mirrors by starting from the fp16-rounded state.

Config 3 also runs its fp16-I/O decay prefix product and Conv1D at full shape
against the oracle (which is pinned bit-for-bit to the reference's own
gdn_cumdecay_f16 / conv): the decay over every sequence, the conv on sampled
sequences.

Bars: 2e-2 relative L2 on outputs and final state (the bf16 / fp16-state
bar); the conv bit-exact; the decay within one fp16 step of the oracle (over
8192 rows the GPU forms the fp32 running product in another association, a
few fp32 ulps apart, which can move a value across one fp16 rounding
boundary).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2
from orionsbelt_b200 import ops, synth

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _pair_inputs(d, b, h, Hv, Hk):
    """Host float32 copies of one (batch, value head) pair, BTHD with one head."""
    hk = h // (Hv // Hk)
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    q = f(d["q"][b:b + 1, :, hk:hk + 1])
    k = f(d["k"][b:b + 1, :, hk:hk + 1])
    v = f(d["v"][b:b + 1, :, h:h + 1])
    g = f(d["g"][b:b + 1, :, h:h + 1])
    beta = f(d["beta"][b:b + 1, :, h:h + 1])
    S0 = f(d["S0"][b:b + 1, h:h + 1])
    return [np.ascontiguousarray(x) for x in (q, k, v, g, beta, S0)]


def _check_pairs(cuda, orc, d, S, o, pairs, Hv, Hk, scale):
    for b, h in pairs:
        q, k, v, g, beta, S0 = _pair_inputs(d, b, h, Hv, Hk)
        S_want, o_want = orc.delta_rule_seq(S0, q, k, v, g, beta, scale=scale)
        o_got = o[b:b + 1, :, h:h + 1].float().cpu().numpy()
        S_got = S[b:b + 1, h:h + 1].float().cpu().numpy()
        eo, es = rel_l2(o_got, o_want), rel_l2(S_got, S_want)
        assert eo < TOL and es < TOL, (b, h, eo, es)


def test_tc_config2_full_vs_oracle(cuda, orc):
    torch = cuda
    B, T, Hk, Hv = 8, 32768, 16, 32
    d = synth.device_gdn(B, T, Hk, Hv, 128, 128, g_scale=0.1, seed=77, in_dtype=torch.bfloat16)
    S = d["S0"].clone()
    o = torch.empty_like(d["v"])
    ops.chunk_delta_rule(d["q"], d["k"], d["v"], d["g"], d["beta"], S, o, scale=1.0)
    torch.cuda.synchronize()
    assert torch.isfinite(o).all() and torch.isfinite(S).all()
    _check_pairs(cuda, orc, d, S, o, [(0, 0), (3, 17), (7, 31)], Hv, Hk, 1.0)


def test_tc_config3_full_vs_oracle(cuda, orc):
    torch = cuda
    B, T, Hk, Hv = 32, 8192, 16, 32
    h16 = torch.float16
    d = synth.device_gdn(B, T, Hk, Hv, 128, 128, g_scale=1.0, seed=14, in_dtype=h16, state_std=0.05,
                         state_dtype=h16)
    S = d["S0"].clone()
    o = torch.empty_like(d["v"])
    ops.chunk_delta_rule(d["q"], d["k"], d["v"], d["g"], d["beta"], S, o, scale=1.0)
    torch.cuda.synchronize()
    assert torch.isfinite(o).all() and torch.isfinite(S).all()
    _check_pairs(cuda, orc, d, S, o, [(0, 1), (13, 8), (31, 30)], Hv, Hk, 1.0)


def test_config3_decay_fp16_full(cuda, orc):
    """Prefix product of a = exp(g) over [32][8192][32], stored as fp16."""
    torch = cuda
    g = -torch.nn.functional.softplus(synth.device_normal((32, 8192, 32), 21, 1))
    a = torch.exp(g).contiguous()
    out = torch.empty(a.shape, dtype=torch.float16, device="cuda")
    ops.cumdecay(a, out)
    got = out.view(torch.int16).cpu().numpy().view(np.uint16)
    ah = a.cpu().numpy()
    for b in range(32):
        want = orc.cumdecay_narrow(np.ascontiguousarray(ah[b]), "f16")
        # positive values: the fp16 encodings order like the numbers
        diff = np.abs(got[b].astype(np.int32) - want.astype(np.int32))
        assert diff.max() <= 1, (b, int(diff.max()))
        assert (diff == 0).mean() > 0.99, b


def test_config3_conv_fp16_full(cuda, orc):
    """Conv1D k4 over [32][8192][8192] fp16 I/O; sampled sequences bit-exact."""
    torch = cuda
    B, T, Cc = 32, 8192, 8192
    x = synth.device_normal((B, T, Cc), 22, 1, dtype=torch.float16)
    w = synth.device_normal((4, Cc), 22, 2, std=0.5)
    hist = synth.device_normal((B, 3, Cc), 22, 3, dtype=torch.float16)
    out = torch.empty_like(x)
    hist_gpu = hist.clone()
    ops.causal_dwconv1d(x, w, out, hist_gpu)
    torch.cuda.synchronize()
    u16 = lambda t: t.view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    wh = w.cpu().numpy()
    for b in (0, 17, 31):
        o_want, h_want = orc.conv_narrow(np.ascontiguousarray(u16(x[b])), wh, np.ascontiguousarray(u16(hist[b])),
                                         "f16")
        assert np.array_equal(u16(out[b]), o_want), b
        assert np.array_equal(u16(hist_gpu[b]), h_want), b
