"""GPU parity of the GDN-2 decode step (decoupled gating: per-key-channel decay,
erase gate b, write gate w; bench/gdn2_reference.py:58-145) through the C ABI
kai_run_gdn2_delta_rule_decode_sm100a, against the oracle's restatement and the
reference's own float64 vectors.

Tolerances (written here, per the build's parity bar):
  fp32 paths                 1e-4 relative L2 on outputs and final state
  bf16 inputs / narrow state 2e-2 relative L2
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import rel_l2
from orionsbelt_b200 import _lib, ops, synth

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-4
NARROW_TOL = 2e-2


def _t(cuda, a, dtype=None):
    t = cuda.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def _round(a, kind):
    if kind == "f32":
        return np.asarray(a, np.float32)
    return oracle.u16_to_f32(oracle.f32_to_u16(a, kind), kind)


def _case(B, Hk, Hv, d, seed, state_std=0.02, g_scale=0.1):
    """Gates as the reference makes them (bench/gdn2_reference.py:224-248):
    g = -softplus(.) per key channel, b and w = sigmoid(.)."""
    r = np.random.default_rng(seed)
    S = (r.standard_normal((B, Hv, d, d)) * state_std).astype(np.float32)
    q = synth.l2norm(r.uniform(-1, 1, (B, Hk, d)))
    k = synth.l2norm(r.uniform(-1, 1, (B, Hk, d)))
    v = r.uniform(-0.5, 0.5, (B, Hv, d)).astype(np.float32)
    g = (-np.log1p(np.exp(r.standard_normal((B, Hv, d)))) * g_scale).astype(np.float32)
    bg = (1 / (1 + np.exp(-r.standard_normal((B, Hv, d))))).astype(np.float32)
    wg = (1 / (1 + np.exp(-r.standard_normal((B, Hv, d))))).astype(np.float32)
    return S, q, k, v, g, bg, wg


def _run(cuda, S, q, k, v, g, bg, wg, scale, in_dt=None, state_dt=None, out_dt=None):
    in_dt = in_dt or cuda.float32
    Sd = _t(cuda, S, state_dt)
    o = cuda.empty(v.shape, dtype=out_dt or cuda.float32, device="cuda")
    ops.gdn2_delta_rule_decode(Sd, _t(cuda, q, in_dt), _t(cuda, k, in_dt), _t(cuda, v, in_dt), _t(cuda, g),
                               _t(cuda, bg), _t(cuda, wg), o, scale=scale)
    return Sd.float().cpu().numpy(), o.float().cpu().numpy()


@pytest.mark.parametrize("B,Hk,Hv,d", [(1, 1, 1, 32), (3, 2, 4, 128), (2, 16, 32, 128), (5, 1, 3, 64),
                                       (4, 2, 2, 32), (64, 16, 32, 128)])
def test_gdn2_decode_fp32(cuda, orc, B, Hk, Hv, d):
    S, q, k, v, g, bg, wg = _case(B, Hk, Hv, d, B * 31 + Hv + d)
    sc = 1.0 / np.sqrt(d)
    S_want, o_want = orc.gdn2_decode(S, q, k, v, g, bg, wg, scale=sc)
    S_got, o_got = _run(cuda, S, q, k, v, g, bg, wg, sc)
    assert rel_l2(o_got, o_want) < FP32_TOL and rel_l2(S_got, S_want) < FP32_TOL


@pytest.mark.parametrize("in_kind,state_kind", [("bf16", "f32"), ("bf16", "bf16"), ("f16", "f16"), ("f32", "bf16")])
def test_gdn2_decode_narrow(cuda, orc, in_kind, state_kind):
    tdt = {"f32": cuda.float32, "bf16": cuda.bfloat16, "f16": cuda.float16}
    S, q, k, v, g, bg, wg = _case(4, 16, 32, 128, 9)
    qr, kr, vr = (_round(x, in_kind) for x in (q, k, v))
    Sr = _round(S, state_kind)
    S_want, o_want = orc.gdn2_decode(Sr, qr, kr, vr, g, bg, wg, scale=1.0)
    S_got, o_got = _run(cuda, Sr, qr, kr, vr, g, bg, wg, 1.0, in_dt=tdt[in_kind], state_dt=tdt[state_kind],
                        out_dt=cuda.bfloat16 if in_kind == "bf16" else cuda.float32)
    tol = FP32_TOL if (state_kind == "f32" and in_kind == "f32") else NARROW_TOL
    assert rel_l2(o_got, o_want) < tol and rel_l2(S_got, S_want) < tol


def test_gdn2_decode_reference_vectors(cuda, golden):
    """The reference's gdn2_recurrent (float64) on grouped heads, T=5 tokens as
    five launches on one state."""
    d = golden("gdn2_general.npz")
    S = _t(cuda, d["S0"][None])
    o = cuda.empty((1, 4, 32), dtype=cuda.float32, device="cuda")
    outs = []
    for t in range(d["q"].shape[0]):
        ops.gdn2_delta_rule_decode(S, _t(cuda, d["q"][t][None]), _t(cuda, d["k"][t][None]),
                                   _t(cuda, d["v"][t][None]), _t(cuda, d["g"][t][None]),
                                   _t(cuda, d["b_gate"][t][None]), _t(cuda, d["w_gate"][t][None]), o,
                                   scale=float(d["scale"]))
        outs.append(o.cpu().numpy()[0])
    assert rel_l2(np.stack(outs), d["o"]) < FP32_TOL
    assert rel_l2(S.cpu().numpy()[0], d["S"]) < FP32_TOL


def test_gdn2_uniform_gates_equal_gdn1_kernel(cuda):
    """Uniform gates (g_j = g, b_j = w_i = beta) make the GDN-2 kernel compute the
    GDN-1 step of kai_run_gdn_delta_rule_decode_sm100a: the reduction of
    bench/gdn2_reference.py:293-349, checked between the two entry points."""
    B, Hk, Hv, d = 8, 4, 8, 128
    S, q, k, v, g, bg, wg = _case(B, Hk, Hv, d, 3)
    g1 = g[..., 0].copy()
    b1 = bg[..., 0].copy()
    gu = np.repeat(g1[..., None], d, -1)
    bu = np.repeat(b1[..., None], d, -1)
    S2, o2 = _run(cuda, S, q, k, v, gu, bu, bu, 0.5)
    S1 = _t(cuda, S)
    o1 = cuda.empty(v.shape, dtype=cuda.float32, device="cuda")
    ops.delta_rule_decode(S1, _t(cuda, q), _t(cuda, k), _t(cuda, v), _t(cuda, g1), _t(cuda, b1), o1, scale=0.5)
    assert rel_l2(o2, o1.cpu().numpy()) < 1e-5 and rel_l2(S2, S1.cpu().numpy()) < 1e-5


def test_gdn2_decode_errors(cuda):
    """Shape checks fail loudly with a status, as the GDN-1 entry does."""
    S, q, k, v, g, bg, wg = _case(1, 1, 1, 96, 1)
    with pytest.raises(_lib.GdnError, match="head dim"):
        _run(cuda, S, q, k, v, g, bg, wg, 1.0)
    _lib.lib().kai_gdn_cuda_clear_error()
    S, q, k, v, g, bg, wg = _case(1, 2, 3, 32, 1)
    with pytest.raises(_lib.GdnError, match="multiple"):
        _run(cuda, S, q, k, v, g, bg, wg, 1.0)
    _lib.lib().kai_gdn_cuda_clear_error()
