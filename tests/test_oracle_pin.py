"""Pin the CPU oracle (oracle/gdn_oracle.c) before trusting it (CPU only).

* Against the reference's own C kernels, compiled from the reference sources
  into oracle/_ref/libgdnref.so: bit-identical on every kernel the reference
  has C code for.
* Against the committed golden fixtures: the reference's NumPy recurrence
  (bench/gdn2_reference.py), its GDN-2 path with uniform gates, HF's chunkwise
  form, and the reference C on the kai test's LCG inputs.
* The chunked-WY restatement against the token loop, and the hand-checkable
  known answer.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2

import oracle


def _need_ref(ref):
    if ref is None:
        pytest.skip("oracle/_ref/libgdnref.so not built (no reference tree at build time)")


SHAPES = [(1, 1), (4, 3), (16, 7), (64, 17), (64, 33), (130, 128), (257, 2051)]


@pytest.mark.parametrize("seq,ch", SHAPES)
def test_channel_kernels_bit_identical_to_reference(orc, ref, seq, ch):
    _need_ref(ref)
    r = np.random.default_rng(seq * 1000 + ch)
    a = r.uniform(0.5, 1.5, (seq, ch)).astype(np.float32)
    assert np.array_equal(orc.cumdecay(a), ref.cumdecay(a))
    assert np.array_equal(orc.cumdecay(a), ref.kai_cumdecay(a))
    for kind in ("f16", "bf16"):
        assert np.array_equal(orc.cumdecay_narrow(a, kind), ref.cumdecay_narrow(a, kind))
    g = r.uniform(-0.99, 0.99, (seq, ch)).astype(np.float32)
    x = r.uniform(-2, 2, (seq, ch)).astype(np.float32)
    st = r.uniform(-1, 1, ch).astype(np.float32)
    s1, st1 = orc.gated_scan(g, x, st)
    s2, st2 = ref.gated_scan(g, x, st)
    assert np.array_equal(s1, s2) and np.array_equal(st1, st2)
    for kind in ("f16", "bf16"):
        stn = oracle.f32_to_u16(st, kind)
        s1, st1 = orc.gated_scan_narrow(g, x, stn, kind)
        s2, st2 = ref.gated_scan_narrow(g, x, stn, kind)
        assert np.array_equal(s1, s2) and np.array_equal(st1, st2)
    w = r.uniform(-1, 1, (4, ch)).astype(np.float32)
    h = r.uniform(-1, 1, (3, ch)).astype(np.float32)
    o1, h1 = orc.conv(x, w, h)
    o2, h2 = ref.conv(x, w, h)
    assert np.array_equal(o1, o2) and np.array_equal(h1, h2)
    bg = r.uniform(0, 1, (seq, ch)).astype(np.float32)
    wg = r.uniform(0, 1, (seq, ch)).astype(np.float32)
    s1, st1 = orc.gdn2_scan(g, bg, wg, x, st)
    s2, st2 = ref.gdn2_scan(g, bg, wg, x, st)
    assert np.array_equal(s1, s2) and np.array_equal(st1, st2)


@pytest.mark.parametrize("M,K,N", [(1, 128, 128), (64, 128, 128), (1, 128, 2048), (64, 128, 130), (5, 7, 3)])
def test_matmul_bit_identical_to_reference(orc, ref, M, K, N):
    _need_ref(ref)
    r = np.random.default_rng(M * 7 + N)
    A = r.uniform(-1, 1, (M, K)).astype(np.float32)
    B = r.uniform(-1, 1, (K, N)).astype(np.float32)
    assert np.array_equal(orc.matmul(A, B), ref.matmul(A, B))
    if M == 1:
        assert np.array_equal(orc.gemv(A[0], B), ref.gemv(A[0], B))


def test_kai_lcg_golden(orc, golden):
    """The reference C on the kai test's own LCG inputs (kai_lcg.npz)."""
    d = golden("kai_lcg.npz")
    assert np.array_equal(orc.cumdecay(d["a"]), d["decay"])
    s, st = orc.gated_scan(d["g"], d["x"], d["s0"])
    assert np.array_equal(s, d["s"]) and np.array_equal(st, d["s_state"])
    o, h = orc.conv(d["cin"], d["w"], d["h0"])
    assert np.array_equal(o, d["conv_out"]) and np.array_equal(h, d["conv_hist"])
    assert np.array_equal(orc.gemv(d["ga"], d["gb"]), d["gemv"])


def test_gdn1_recurrent_golden(orc, golden):
    """bench/gdn2_reference.py::gdn1_recurrent (float64) on grouped heads."""
    d = golden("gdn1_recurrent.npz")
    S, o = orc.delta_rule_seq(d["S0"], d["q"], d["k"], d["v"], d["g"], d["beta"], scale=float(d["scale"]))
    assert rel_l2(o[0], d["o"]) < 1e-5
    assert rel_l2(S[0], d["S"]) < 1e-5


def test_gdn2_uniform_golden(orc, golden):
    """The reference's GDN-2 recurrence with uniform gates equals GDN-1 with beta."""
    d = golden("gdn2_uniform.npz")
    S, o = orc.delta_rule_seq(d["S0"], d["q"], d["k"], d["v"], d["g"], d["beta"], scale=1.0)
    assert rel_l2(o[0], d["o"]) < 1e-5
    assert rel_l2(S[0], d["S"]) < 1e-5


def test_hf_chunk_golden(orc, golden):
    """HF torch_chunk_gated_delta_rule (chunked WY, fp32) vs both oracle forms."""
    d = golden("hf_chunk.npz")
    sc = float(d["scale"])
    S, o = orc.delta_rule_seq(d["S0"], d["q"], d["k"], d["v"], d["g"], d["beta"], scale=sc)
    assert rel_l2(o, d["o"]) < 1e-5 and rel_l2(S, d["S"]) < 1e-5
    S2, o2 = orc.chunk_wy(d["S0"], d["q"], d["k"], d["v"], d["g"], d["beta"], scale=sc)
    assert rel_l2(o2, d["o"]) < 1e-5 and rel_l2(S2, d["S"]) < 1e-5


@pytest.mark.parametrize("T", [1, 63, 64, 65, 130])
def test_chunk_wy_equals_token_loop(orc, T):
    from orionsbelt_b200 import synth
    d = synth.host_gdn(1, T, 2, 4, 16, 16, g_scale=1.0, seed=T, state_std=0.2)
    S1, o1 = orc.delta_rule_seq(d["S0"], d["q"], d["k"], d["v"], d["g"], d["beta"], scale=0.25)
    S2, o2 = orc.chunk_wy(d["S0"], d["q"], d["k"], d["v"], d["g"], d["beta"], scale=0.25)
    assert rel_l2(o2, o1) < 1e-5 and rel_l2(S2, S1) < 1e-5


def test_known_answer(orc):
    """T=1, dk=dv=2, S0=0, beta=1: S = k v^T, o = S^T q (hand-computed, in the
    spirit of bench/gdn2_reference.py:251-290)."""
    k = np.array([0.8, 0.6], np.float32)
    v = np.array([1.0, 2.0], np.float32)
    q = np.array([0.6, 0.8], np.float32)
    S, o = orc.delta_rule_step(np.zeros((2, 2), np.float32), k, v, q, 1.0, 0.5)
    assert np.allclose(S, [[0.8, 1.6], [0.6, 1.2]], atol=1e-7)
    assert np.allclose(o, [0.96, 1.92], atol=1e-6)
    # beta = 0: no write, only decay (tests/test_gdn2_reference.py:212 analogue)
    S0 = np.array([[1.0, 2.0], [3.0, 4.0]], np.float32)
    S, o = orc.delta_rule_step(S0, k, v, q, 0.0, 0.5)
    assert np.array_equal(S, S0 * np.float32(0.5))


def test_integer_inputs_exact(orc):
    """Conv and cumsum are exact on integer-valued inputs."""
    r = np.random.default_rng(5)
    x = r.integers(-3, 4, (100, 9)).astype(np.float32)
    w = r.integers(-3, 4, (4, 9)).astype(np.float32)
    h = r.integers(-3, 4, (3, 9)).astype(np.float32)
    o, _ = orc.conv(x, w, h)
    full = np.concatenate([h, x]).astype(np.int64)
    want = sum(w[j].astype(np.int64) * full[j:j + 100] for j in range(4))
    assert np.array_equal(o.astype(np.int64), want)
    g = r.integers(-3, 1, (100, 9)).astype(np.float32)
    assert np.array_equal(orc.cumsum(g).astype(np.int64), np.cumsum(g.astype(np.int64), axis=0))


def test_gdn2_general_golden(orc, golden):
    """bench/gdn2_reference.py::gdn2_recurrent (float64) with per-channel decay,
    erase and write gates on grouped heads, token by token through the oracle."""
    d = golden("gdn2_general.npz")
    sc = float(d["scale"])
    S = d["S0"][None]
    for t in range(d["q"].shape[0]):
        S, o = orc.gdn2_decode(S, d["q"][t][None], d["k"][t][None], d["v"][t][None], d["g"][t][None],
                               d["b_gate"][t][None], d["w_gate"][t][None], scale=sc)
        o_t = o[0]
    assert rel_l2(o_t, d["o"][-1]) < 1e-5
    assert rel_l2(S[0], d["S"]) < 1e-5
    T = d["q"].shape[0]
    S2, o2 = orc.gdn2_seq(d["S0"][None], d["q"][None], d["k"][None], d["v"][None], d["g"][None],
                          d["b_gate"][None], d["w_gate"][None], scale=sc)
    assert rel_l2(o2[0], d["o"]) < 1e-5 and rel_l2(S2[0], d["S"]) < 1e-5
    assert o2.shape == (1, T, 4, 32)


def test_gdn2_uniform_gates_equal_gdn1(orc, golden):
    """GDN-2 with g_j = g, b_j = w_i = beta is GDN-1 (the reduction the reference
    tests at bench/gdn2_reference.py:293-349), on its uniform-gate vectors."""
    d = golden("gdn2_uniform.npz")
    B, T, Hv = d["g"].shape
    dk, dv = d["k"].shape[-1], d["v"].shape[-1]
    g = np.repeat(d["g"][..., None], dk, -1)
    bg = np.repeat(d["beta"][..., None], dk, -1)
    wg = np.repeat(d["beta"][..., None], dv, -1)
    S, o = orc.gdn2_seq(d["S0"], d["q"], d["k"], d["v"], g, bg, wg, scale=1.0)
    assert rel_l2(o[0], d["o"]) < 1e-5 and rel_l2(S[0], d["S"]) < 1e-5


def test_gdn2_known_answer(orc):
    """dk = dv = 2 by hand.  From S0 = 0 only the write gate acts: S = k (w v)^T.
    With w = 0 only decay and erase act: S = D S0 - k (S0^T D (b k))^T."""
    k = np.array([[[0.8, 0.6]]], np.float32)
    q = np.array([[[0.6, 0.8]]], np.float32)
    v = np.array([[[1.0, 2.0]]], np.float32)
    S, o = orc.gdn2_decode(np.zeros((1, 1, 2, 2), np.float32), q, k, v, np.zeros((1, 1, 2), np.float32),
                           np.ones((1, 1, 2), np.float32), np.array([[[0.5, 1.0]]], np.float32))
    assert np.allclose(S[0, 0], [[0.4, 1.6], [0.3, 1.2]], atol=1e-7)
    assert np.allclose(o[0, 0], [0.48, 1.92], atol=1e-6)
    S0 = np.array([[[[1.0, 2.0], [3.0, 4.0]]]], np.float32)
    S, o = orc.gdn2_decode(S0, q, k, v, np.log(np.array([[[0.5, 1.0]]], np.float32)),
                           np.array([[[1.0, 0.0]]], np.float32), np.zeros((1, 1, 2), np.float32))
    assert np.allclose(S[0, 0], [[0.18, 0.36], [2.76, 3.52]], atol=1e-6)
    assert np.allclose(o[0, 0], [2.316, 3.032], atol=1e-5)


@pytest.mark.parametrize("K,N", [(128, 256), (64, 130), (2560, 1024), (7, 3)])
def test_int8_bit_identical_to_reference(orc, K, N):
    """quantize_weight, gemv_int8_neon and gemm_int8_neon (gdn_e2e_decode.c:175,
    296, 608; built from the reference tree by oracle/ref_int8_shim.c) against
    the oracle: same codes, scales and outputs, bit for bit.  Includes an
    all-zero column (scale 1), ragged N and values on a rounding tie."""
    import oracle
    if oracle.ref_int8 is None:
        pytest.skip("oracle/_ref/libint8ref.so not built (needs the reference tree)")
    r = np.random.default_rng(K * 7 + N)
    B = r.uniform(-1, 1, (K, N)).astype(np.float32)
    B[:, 0] = 0.0
    if N > 2:
        B[0, 2], B[1, 2] = 1.0, 0.5 / 127.0  # q = 127 and a half-way code
    q1, s1 = orc.quantize_int8(B)
    q2, s2 = oracle.ref_int8.quantize_int8(B)
    assert np.array_equal(q1, q2) and np.array_equal(s1, s2)
    for M in (1, 3):
        A = r.uniform(-1, 1, (M, K)).astype(np.float32)
        assert np.array_equal(orc.matmul_int8(A, q1, s1), oracle.ref_int8.matmul_int8(A, q1, s1))


def test_int8_reference_accuracy_rules(orc):
    """The reference test's own rules on the oracle (test_gdn_e2e_int8.c:57-161):
    scale = max|col| / 127, |C - A.B| <= s * 0.5 * sum|a| (x2 margin), mean
    relative error < 2% where |A.B| > 1."""
    r = np.random.default_rng(42)
    K, N = 128, 256
    W = r.uniform(-1, 1, (K, N)).astype(np.float32)
    q, s = orc.quantize_int8(W)
    assert np.allclose(s, np.abs(W).max(0) / np.float32(127), rtol=1e-6, atol=0)
    a = r.uniform(-1, 1, (1, K)).astype(np.float32)
    c = orc.matmul_int8(a, q, s)[0]
    c32 = (a.astype(np.float64) @ W.astype(np.float64))[0]
    bound = s.astype(np.float64) * 0.5 * np.abs(a).sum()
    assert (np.abs(c - c32) <= 2 * bound).all()
    big = np.abs(c32) > 1.0
    assert np.mean(np.abs(c[big] - c32[big]) / np.abs(c32[big])) < 0.02


@pytest.mark.parametrize("pos,max_ctx", [(0, 1), (37, 64), (300, 301)])
@pytest.mark.parametrize("kind", ["f32", "i8"])
def test_attn_decode_bit_identical_to_reference(orc, pos, max_ctx, kind):
    """The reference's own GQA attention decode (gdn_e2e_decode.c:1532-1634
    full_attn_real_forward and, built with KV_INT8, :1652-1830
    full_attn_real_forward_int8kv; run through oracle/ref_attn_shim.c) against
    the oracle: same outputs and same appended cache entries, bit for bit."""
    import oracle
    ra = oracle.ref_attn if kind == "f32" else oracle.ref_attn_i8
    if ra is None:
        pytest.skip("oracle/_ref attention shims not built (need the reference tree)")
    H, Hkv, D = ra.heads, ra.kv_heads, ra.head_dim
    r = np.random.default_rng(pos + (7 if kind == "i8" else 0))
    q = r.uniform(-1, 1, H * D).astype(np.float32)
    kn, vn = (r.uniform(-1, 1, Hkv * D).astype(np.float32) for _ in range(2))
    if kind == "f32":
        kc, vc = (r.uniform(-1, 1, (max_ctx, Hkv * D)).astype(np.float32) for _ in range(2))
        ks = vs = None
    else:
        kc, vc = (r.integers(-128, 128, (max_ctx, Hkv * D)).astype(np.int8) for _ in range(2))
        ks, vs = (r.uniform(0.001, 0.02, Hkv).astype(np.float32) for _ in range(2))
    kc2, vc2 = kc.copy(), vc.copy()
    o_ref = ra.attn_decode(q, kn, vn, kc, vc, pos, ks, vs)
    o = orc.attn_decode(q.reshape(1, H, D), kn.reshape(1, Hkv, D), vn.reshape(1, Hkv, D),
                        kc2.reshape(1, max_ctx, Hkv, D), vc2.reshape(1, max_ctx, Hkv, D), pos,
                        1.0 / np.sqrt(np.float32(D)), None if ks is None else ks[None],
                        None if vs is None else vs[None])
    assert np.array_equal(o.ravel(), o_ref)
    assert np.array_equal(kc2, kc) and np.array_equal(vc2, vc)


def e2e_weights(dims, seed, sigma=0.007):
    """Seeded weights for the end-to-end loop: projections N(0, sigma) (one set
    serves every layer, so larger weights overflow within a few layers), conv
    weights N(0, 1/4), gates U(0, 1)."""
    import oracle
    shapes = oracle.e2e_weight_shapes(dims)
    r = np.random.default_rng(seed)
    W = {n: (r.standard_normal(s) * sigma).astype(np.float32) for n, s in shapes.items()}
    W["g_conv_w"] = (r.standard_normal(shapes["g_conv_w"]) * 0.5).astype(np.float32)
    W["g_beta"] = r.uniform(0, 1, shapes["g_beta"]).astype(np.float32)
    return W


def test_e2e_decode_bit_identical_to_reference(orc):
    """The reference's own end-to-end decode loop (gdn_e2e_decode.c:2775-2796,
    INT8_WEIGHTS, 0.8B geometry; run through oracle/ref_e2e_shim.c) against the
    oracle over three tokens: same hidden outputs and GDN states, bit for bit."""
    import oracle
    if oracle.ref_e2e is None:
        pytest.skip("oracle/_ref/libe2eref.so not built (needs the reference tree)")
    dims = oracle.ref_e2e.dims
    W = e2e_weights(dims, 0)
    hin = np.random.default_rng(1).standard_normal((3, dims[0])).astype(np.float32)
    o_ref, st_ref = oracle.ref_e2e.e2e_decode(W, hin)
    o, st = orc.e2e_decode(dims, oracle.e2e_layer_pattern(dims[8]), W, hin[:, None, :])
    assert np.isfinite(o_ref).all()
    assert np.array_equal(o[:, 0], o_ref) and np.array_equal(st[:, 0], st_ref)
