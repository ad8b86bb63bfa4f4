"""GPU parity of the matrix-state delta rule: the decode step (config 1) and
the chunkwise WY scan (configs 0, 2, 3), through the C ABI, against the
oracle's restatement of gpu/gdn_gpu_validate.c:100-118 and its token loop.

Tolerances (written here, per the build's parity bar):
  fp32 paths            1e-4 relative L2 on outputs and final state
  bf16 inputs / fp16 state  2e-2 relative L2
plus the reference's own pass rule of gpu/gdn_gpu_validate.c:145 on the
decode cases it tests (dims 32-128, beta in {0, 1}, decay in {0.01, 0.99, 1}).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import rel_l2, validate_pass
from orionsbelt_b200 import ops, synth

pytestmark = pytest.mark.gpu

FP32_TOL = 1e-4
NARROW_TOL = 2e-2


def _t(cuda, a, dtype=None):
    t = cuda.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def _round(a, kind):
    """Round fp32 values through a narrow format (what the GPU sees)."""
    if kind == "f32":
        return np.asarray(a, np.float32)
    return oracle.u16_to_f32(oracle.f32_to_u16(a, "f16" if kind == "f16" else "bf16"), "f16" if kind == "f16" else "bf16")


# ------------------------------------------------------------------ decode

def _decode_case(B, Hk, Hv, d, seed, beta=None, decay=None, state_std=0.01):
    r = np.random.default_rng(seed)
    S = (r.uniform(-1, 1, (B, Hv, d, d)) * state_std).astype(np.float32)
    q = synth.l2norm(r.uniform(-1, 1, (B, Hk, d)))
    k = synth.l2norm(r.uniform(-1, 1, (B, Hk, d)))
    v = r.uniform(-0.5, 0.5, (B, Hv, d)).astype(np.float32)
    b = np.full((B, Hv), beta, np.float32) if beta is not None else r.uniform(0, 1, (B, Hv)).astype(np.float32)
    g = (np.full((B, Hv), np.log(decay), np.float32) if decay is not None
         else -np.log1p(np.exp(r.standard_normal((B, Hv)))).astype(np.float32) * 0.1)
    return S, q, k, v, g.astype(np.float32), b


def _run_decode(cuda, S, q, k, v, g, b, scale, in_dt=None, state_dt=None, out_dt=None):
    in_dt = in_dt or cuda.float32
    Sd = _t(cuda, S, state_dt)
    o = cuda.empty(v.shape, dtype=out_dt or cuda.float32, device="cuda")
    ops.delta_rule_decode(Sd, _t(cuda, q, in_dt), _t(cuda, k, in_dt), _t(cuda, v, in_dt), _t(cuda, g), _t(cuda, b),
                          o, scale=scale)
    return Sd.float().cpu().numpy(), o.float().cpu().numpy()


VALIDATE_CASES = [  # gpu/gdn_gpu_validate.c:623-640
    ("delta_0.8B", 16, 128, 0.5, 0.9), ("delta_4B_32heads", 32, 128, 0.5, 0.9),
    ("delta_decay_0.01", 16, 128, 0.5, 0.01), ("delta_decay_0.99", 16, 128, 0.5, 0.99),
    ("delta_decay_1.0", 16, 128, 0.5, 1.0), ("delta_beta_0", 16, 128, 0.0, 0.9),
    ("delta_beta_1", 16, 128, 1.0, 0.9), ("delta_64x64", 8, 64, 0.5, 0.9), ("delta_32x32", 4, 32, 0.5, 0.9),
]


@pytest.mark.parametrize("name,H,d,beta,decay", VALIDATE_CASES)
def test_decode_reference_validation_cases(cuda, orc, name, H, d, beta, decay):
    S, q, k, v, g, b = _decode_case(1, H, H, d, hash(name) % 1000, beta=beta, decay=decay)
    S_want, o_want = orc.delta_rule_decode(S, q, k, v, g, b, scale=1.0)
    S_got, o_got = _run_decode(cuda, S, q, k, v, g, b, 1.0)
    assert validate_pass(o_got, o_want) and validate_pass(S_got, S_want), name
    assert rel_l2(o_got, o_want) < FP32_TOL and rel_l2(S_got, S_want) < FP32_TOL


@pytest.mark.parametrize("B,Hk,Hv,d", [(3, 2, 4, 128), (2, 16, 32, 128), (5, 1, 3, 64), (4, 2, 2, 32)])
def test_decode_grouped_heads_fp32(cuda, orc, B, Hk, Hv, d):
    S, q, k, v, g, b = _decode_case(B, Hk, Hv, d, B * 100 + Hv, state_std=0.02)
    sc = 1.0 / np.sqrt(d)
    S_want, o_want = orc.delta_rule_decode(S, q, k, v, g, b, scale=sc)
    S_got, o_got = _run_decode(cuda, S, q, k, v, g, b, sc)
    assert rel_l2(o_got, o_want) < FP32_TOL and rel_l2(S_got, S_want) < FP32_TOL


@pytest.mark.parametrize("in_kind,state_kind", [("bf16", "f32"), ("bf16", "f16"), ("f16", "bf16"), ("f32", "f16")])
def test_decode_narrow(cuda, orc, in_kind, state_kind):
    """Config-1 dtypes (bf16 q/k/v) and narrow state storage: the oracle gets
    the same rounded inputs, widened; the result is compared at 2e-2."""
    tdt = {"f32": cuda.float32, "bf16": cuda.bfloat16, "f16": cuda.float16}
    S, q, k, v, g, b = _decode_case(4, 16, 32, 128, 7, state_std=0.02)
    qr, kr, vr = (_round(x, in_kind) for x in (q, k, v))
    Sr = _round(S, state_kind)
    S_want, o_want = orc.delta_rule_decode(Sr, qr, kr, vr, g, b, scale=1.0)
    S_got, o_got = _run_decode(cuda, Sr, qr, kr, vr, g, b, 1.0, in_dt=tdt[in_kind], state_dt=tdt[state_kind],
                               out_dt=cuda.bfloat16 if in_kind == "bf16" else cuda.float32)
    tol = FP32_TOL if (state_kind == "f32" and in_kind == "f32") else NARROW_TOL
    assert rel_l2(o_got, o_want) < tol and rel_l2(S_got, S_want) < tol


def test_decode_config1_layer_against_torch_fp32(cuda):
    """One full config-1 layer (B=64, Hv=32, 128x128, bf16 q/k/v, fp32 state
    N(0, 0.02)) against a plain torch fp32 restatement of the same step."""
    torch = cuda
    d = synth.device_gdn(64, 1, 16, 32, 128, 128, g_scale=0.1, seed=21, in_dtype=torch.bfloat16, state_std=0.02)
    q, k, v = d["q"][:, 0], d["k"][:, 0], d["v"][:, 0]
    g, b, S = d["g"][:, 0].contiguous(), d["beta"][:, 0].contiguous(), d["S0"]
    S_ref = S.clone()
    o = torch.empty((64, 32, 128), dtype=torch.float32, device="cuda")
    ops.delta_rule_decode(S, q.contiguous(), k.contiguous(), v.contiguous(), g, b, o, scale=1.0)
    qf = q.float().repeat_interleave(2, 1)
    kf = k.float().repeat_interleave(2, 1)
    S_ref = S_ref * torch.exp(g)[..., None, None]
    kv = torch.einsum("bhjd,bhj->bhd", S_ref, kf)
    delta = (v.float() - kv) * b[..., None]
    S_ref = S_ref + kf[..., :, None] * delta[..., None, :]
    o_ref = torch.einsum("bhjd,bhj->bhd", S_ref, qf)
    assert (torch.linalg.norm(o - o_ref) / torch.linalg.norm(o_ref)).item() < FP32_TOL
    assert (torch.linalg.norm(S - S_ref) / torch.linalg.norm(S_ref)).item() < FP32_TOL


# ------------------------------------------------------------------- chunk

def _run_chunk(cuda, d, scale, in_dt=None, state_dt=None, out_dt=None):
    in_dt = in_dt or cuda.float32
    S = _t(cuda, d["S0"], state_dt)
    o = cuda.empty(d["v"].shape, dtype=out_dt or cuda.float32, device="cuda")
    ops.chunk_delta_rule(_t(cuda, d["q"], in_dt), _t(cuda, d["k"], in_dt), _t(cuda, d["v"], in_dt), _t(cuda, d["g"]),
                         _t(cuda, d["beta"]), S, o, scale=scale)
    return S.float().cpu().numpy(), o.float().cpu().numpy()


@pytest.mark.parametrize("B,T,Hk,Hv,d", [(1, 1, 1, 1, 128), (1, 63, 2, 4, 128), (1, 64, 2, 4, 128),
                                         (2, 65, 2, 4, 64), (1, 200, 1, 2, 32), (2, 130, 2, 2, 128)])
def test_chunk_fp32_vs_token_loop(cuda, orc, B, T, Hk, Hv, d):
    dd = synth.host_gdn(B, T, Hk, Hv, d, d, g_scale=0.3, seed=T + d, state_std=0.05)
    sc = 1.0 / np.sqrt(d)
    S_want, o_want = orc.delta_rule_seq(dd["S0"], dd["q"], dd["k"], dd["v"], dd["g"], dd["beta"], scale=sc)
    S_got, o_got = _run_chunk(cuda, dd, sc)
    assert rel_l2(o_got, o_want) < FP32_TOL and rel_l2(S_got, S_want) < FP32_TOL


def test_chunk_hf_golden(cuda, golden):
    """HF torch_chunk_gated_delta_rule fixture (ragged last chunk, grouped heads)."""
    d = golden("hf_chunk.npz")
    S_got, o_got = _run_chunk(cuda, d, float(d["scale"]))
    assert rel_l2(o_got, d["o"]) < FP32_TOL and rel_l2(S_got, d["S"]) < FP32_TOL


def test_chunk_config0_full(cuda, orc):
    """Config 0: B=1, T=2048, 16/32 heads, 128x128, fp32 throughout, S0 = 0."""
    c = synth.CONFIGS[0]
    dd = synth.host_gdn(c["B"], c["T"], c["Hk"], c["Hv"], c["dk"], c["dv"], g_scale=c["g_scale"], seed=0)
    S_want, o_want = orc.delta_rule_seq(dd["S0"], dd["q"], dd["k"], dd["v"], dd["g"], dd["beta"], scale=1.0)
    S_got, o_got = _run_chunk(cuda, dd, 1.0)
    assert rel_l2(o_got, o_want) < FP32_TOL and rel_l2(S_got, S_want) < FP32_TOL


@pytest.mark.parametrize("in_kind,state_kind,g_scale", [("bf16", "f32", 0.1), ("bf16", "f16", 1.0), ("f16", "f32", 0.1)])
def test_chunk_narrow(cuda, orc, in_kind, state_kind, g_scale):
    """Config 2 (bf16 q/k/v, fp32 state) and config 3 (fp16 state, strong
    decay) numerics on a shard, at 2e-2."""
    tdt = {"f32": cuda.float32, "bf16": cuda.bfloat16, "f16": cuda.float16}
    dd = synth.host_gdn(2, 300, 2, 4, 128, 128, g_scale=g_scale, seed=31, state_std=0.02)
    for key in ("q", "k", "v"):
        dd[key] = _round(dd[key], in_kind)
    dd["S0"] = _round(dd["S0"], state_kind)
    S_want, o_want = orc.delta_rule_seq(dd["S0"], dd["q"], dd["k"], dd["v"], dd["g"], dd["beta"], scale=1.0)
    S_got, o_got = _run_chunk(cuda, dd, 1.0, in_dt=tdt[in_kind], state_dt=tdt[state_kind], out_dt=tdt[in_kind])
    assert rel_l2(o_got, o_want) < NARROW_TOL and rel_l2(S_got, S_want) < NARROW_TOL


def test_chunk_continuity(cuda, orc):
    """Two chunked calls with the state carried == one call (prefill in pieces,
    the cross-call continuity of kai_gdn_gated_scan_f32_sve.h:26-32)."""
    dd = synth.host_gdn(1, 256, 2, 4, 64, 64, g_scale=0.2, seed=41, state_std=0.05)
    S_full, o_full = _run_chunk(cuda, dd, 0.125)
    first = {k_: (v_[:, :128] if k_ != "S0" else v_) for k_, v_ in dd.items()}
    S_mid, o_a = _run_chunk(cuda, first, 0.125)
    second = {k_: (v_[:, 128:] if k_ != "S0" else S_mid) for k_, v_ in dd.items()}
    S_end, o_b = _run_chunk(cuda, second, 0.125)
    assert rel_l2(np.concatenate([o_a, o_b], 1), o_full) < 1e-5 and rel_l2(S_end, S_full) < 1e-5


def test_chunk_matches_decode_steps(cuda):
    """The chunked scan equals T decode-step launches (same C ABI)."""
    torch = cuda
    d = synth.device_gdn(2, 70, 2, 4, 128, 128, g_scale=0.2, seed=51, state_std=0.02)
    S_c = d["S0"].clone()
    o_c = torch.empty_like(d["v"])
    ops.chunk_delta_rule(d["q"], d["k"], d["v"], d["g"], d["beta"], S_c, o_c, scale=0.5)
    S_d = d["S0"].clone()
    o_d = torch.empty_like(d["v"])
    for t in range(70):
        o_t = torch.empty((2, 4, 128), device="cuda")
        ops.delta_rule_decode(S_d, d["q"][:, t].contiguous(), d["k"][:, t].contiguous(), d["v"][:, t].contiguous(),
                              d["g"][:, t].contiguous(), d["beta"][:, t].contiguous(), o_t, scale=0.5)
        o_d[:, t] = o_t
    rl = lambda a, b: (torch.linalg.norm(a - b) / torch.linalg.norm(b)).item()  # noqa: E731
    assert rl(o_c, o_d) < FP32_TOL and rl(S_c, S_d) < FP32_TOL
