"""GPU parity of the channel-wise operators against the oracle (bit-exact
where the operation order is the reference's).

cumdecay / cumsum / gated scan / GDN-2 scan: a thread walks up to 128 rows in
the reference's order, so seq <= 128 is bit-identical to the reference's
scalar path; longer sequences combine per-segment carries and are checked
with the reference's own tolerances (test_kai_gdn.c:190,222;
gdn_gpu_validate.c:145).  Conv and the matmul are bit-identical at every size.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import kai_close, rel_l2, validate_pass
from orionsbelt_b200 import ops

pytestmark = pytest.mark.gpu

SHORT = [(1, 1), (4, 3), (16, 17), (64, 33), (64, 2051), (128, 129), (1, 8192)]
LONG = [(129, 7), (1024, 32), (4096, 2048), (2048, 32), (32768, 32)]


def _t(cuda, a):
    return cuda.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("seq,ch", SHORT + LONG)
def test_cumdecay(cuda, orc, seq, ch):
    r = np.random.default_rng(seq + ch)
    a = r.uniform(0.9, 1.1, (seq, ch)).astype(np.float32) if seq > 128 else r.uniform(0.5, 1.5, (seq, ch)).astype(np.float32)
    want = orc.cumdecay(a)
    out = cuda.empty((seq, ch), dtype=cuda.float32, device="cuda")
    ops.cumdecay(_t(cuda, a), out)
    got = out.cpu().numpy()
    if seq <= 128:
        assert np.array_equal(got, want)
    else:
        assert kai_close(got, want, 1e-5, 1e-4)


@pytest.mark.parametrize("kind", ["f16", "bf16"])
@pytest.mark.parametrize("seq,ch", [(64, 2051), (7, 5)])
def test_cumdecay_narrow(cuda, orc, kind, seq, ch):
    a = np.random.default_rng(1).uniform(0.5, 0.99, (seq, ch)).astype(np.float32)
    want = orc.cumdecay_narrow(a, kind)
    out = cuda.empty((seq, ch), dtype=cuda.float16 if kind == "f16" else cuda.bfloat16, device="cuda")
    ops.cumdecay(_t(cuda, a), out)
    assert np.array_equal(out.view(cuda.int16).cpu().numpy().view(np.uint16), want)


@pytest.mark.parametrize("seq,ch", SHORT + LONG)
def test_cumsum(cuda, orc, seq, ch):
    g = (-np.log1p(np.exp(np.random.default_rng(seq).standard_normal((seq, ch))))).astype(np.float32)
    want = orc.cumsum(g)
    out = cuda.empty((seq, ch), dtype=cuda.float32, device="cuda")
    ops.cumsum(_t(cuda, g), out)
    got = out.cpu().numpy()
    if seq <= 128:
        assert np.array_equal(got, want)
    else:
        # float sums of up to 32768 terms in two association orders
        assert rel_l2(got, want) < 1e-5


def test_cumsum_integer_exact_batched(cuda):
    """Integer-valued log-decays: exact at config-2 length, batched."""
    r = np.random.default_rng(3)
    g = r.integers(-3, 1, (3, 32768, 32)).astype(np.float32)
    out = cuda.empty(g.shape, dtype=cuda.float32, device="cuda")
    ops.cumsum(_t(cuda, g), out)
    assert np.array_equal(out.cpu().numpy().astype(np.int64), np.cumsum(g.astype(np.int64), axis=1))


def test_cumdecay_power_of_two_exact(cuda, orc):
    """a in {0.5, 1, 2} (exponent walk kept in range): any association is exact."""
    r = np.random.default_rng(4)
    a = r.choice(np.array([0.5, 1.0, 1.0, 1.0, 2.0], np.float32), (2000, 32))
    out = cuda.empty(a.shape, dtype=cuda.float32, device="cuda")
    ops.cumdecay(_t(cuda, a), out)
    assert np.array_equal(out.cpu().numpy(), orc.cumdecay(a))


@pytest.mark.parametrize("seq,ch", SHORT + LONG)
def test_gated_scan(cuda, orc, seq, ch):
    r = np.random.default_rng(seq * 3 + ch)
    g = r.uniform(0.5, 0.9, (seq, ch)).astype(np.float32)
    x = (r.uniform(0, 1, (seq, ch)) - 0.5).astype(np.float32)
    st = r.uniform(-1, 1, ch).astype(np.float32)
    s_want, st_want = orc.gated_scan(g, x, st)
    s = cuda.empty((seq, ch), dtype=cuda.float32, device="cuda")
    st_d = _t(cuda, st)
    ops.gated_scan(_t(cuda, g), _t(cuda, x), s, st_d)
    if seq <= 128:
        assert np.array_equal(s.cpu().numpy(), s_want)
        assert np.array_equal(st_d.cpu().numpy(), st_want)
    else:
        assert validate_pass(s.cpu().numpy(), s_want) and validate_pass(st_d.cpu().numpy(), st_want)


# Long chains: more than 256 tiles of 256 rows per chain, a ragged last
# channel tile, and inputs larger than 64 MiB.
LONG_CHAINS = [
    ("cumsum", 65536, 32),
    ("cumsum", 65537, 32),
    ("cumdecay", 70000, 40),
    ("gated", 65537, 33),
    ("gated", 9000, 1000),
]


@pytest.mark.parametrize("op,seq,ch", LONG_CHAINS)
def test_scan_long_chains(cuda, orc, op, seq, ch):
    r = np.random.default_rng(seq + ch)
    if op == "cumsum":
        g = (-np.log1p(np.exp(r.standard_normal((seq, ch))))).astype(np.float32)
        out = cuda.empty((seq, ch), dtype=cuda.float32, device="cuda")
        ops.cumsum(_t(cuda, g), out)
        assert rel_l2(out.cpu().numpy(), orc.cumsum(g)) < 1e-5
    elif op == "cumdecay":
        a = r.uniform(0.999, 1.001, (seq, ch)).astype(np.float32)  # the product stays in range at 70000 rows
        out = cuda.empty((seq, ch), dtype=cuda.float32, device="cuda")
        ops.cumdecay(_t(cuda, a), out)
        assert kai_close(out.cpu().numpy(), orc.cumdecay(a), 1e-5, 1e-4)
    else:
        g = r.uniform(0.5, 0.99, (seq, ch)).astype(np.float32)
        x = (r.uniform(0, 1, (seq, ch)) - 0.5).astype(np.float32)
        st = r.uniform(-1, 1, ch).astype(np.float32)
        s_want, st_want = orc.gated_scan(g, x, st)
        s = cuda.empty((seq, ch), dtype=cuda.float32, device="cuda")
        st_d = _t(cuda, st)
        ops.gated_scan(_t(cuda, g), _t(cuda, x), s, st_d)
        assert validate_pass(s.cpu().numpy(), s_want) and validate_pass(st_d.cpu().numpy(), st_want)


@pytest.mark.parametrize("kind", ["f16", "bf16"])
def test_gated_scan_narrow_state(cuda, orc, kind):
    seq, ch = 64, 2051
    r = np.random.default_rng(9)
    g = r.uniform(0.5, 0.9, (seq, ch)).astype(np.float32)
    x = (r.uniform(0, 1, (seq, ch)) - 0.5).astype(np.float32)
    st = oracle.f32_to_u16(r.uniform(-0.5, 0.5, ch), kind)
    s_want, st_want = orc.gated_scan_narrow(g, x, st, kind)
    s = cuda.empty((seq, ch), dtype=cuda.float32, device="cuda")
    st_d = cuda.from_numpy(st.view(np.int16).copy()).cuda().view(cuda.float16 if kind == "f16" else cuda.bfloat16)
    ops.gated_scan(_t(cuda, g), _t(cuda, x), s, st_d)
    assert np.array_equal(s.cpu().numpy(), s_want)
    assert np.array_equal(st_d.view(cuda.int16).cpu().numpy().view(np.uint16), st_want)


def test_gated_scan_batched_and_continuity(cuda, orc):
    """Batched call == per-sequence calls; two calls carry state like one."""
    B, T, C = 3, 300, 40
    r = np.random.default_rng(10)
    g = r.uniform(0.5, 0.99, (B, T, C)).astype(np.float32)
    x = r.uniform(-2, 2, (B, T, C)).astype(np.float32)
    st = r.uniform(-1, 1, (B, C)).astype(np.float32)
    s = cuda.empty((B, T, C), dtype=cuda.float32, device="cuda")
    st_d = _t(cuda, st)
    ops.gated_scan(_t(cuda, g), _t(cuda, x), s, st_d)
    for b in range(B):
        s_want, st_want = orc.gated_scan(g[b], x[b], st[b])
        assert validate_pass(s[b].cpu().numpy(), s_want)
        assert validate_pass(st_d[b].cpu().numpy(), st_want)
    # continuity at the bit level for short calls: 8 + 8 == 16
    g1, x1, st1 = g[0, :16], x[0, :16], st[0]
    s_want, st_want = orc.gated_scan(g1, x1, st1)
    st_d = _t(cuda, st1)
    s_a = cuda.empty((8, C), dtype=cuda.float32, device="cuda")
    s_b = cuda.empty((8, C), dtype=cuda.float32, device="cuda")
    ops.gated_scan(_t(cuda, g1[:8]), _t(cuda, x1[:8]), s_a, st_d)
    ops.gated_scan(_t(cuda, g1[8:]), _t(cuda, x1[8:]), s_b, st_d)
    assert np.array_equal(np.concatenate([s_a.cpu().numpy(), s_b.cpu().numpy()]), s_want)
    assert np.array_equal(st_d.cpu().numpy(), st_want)


@pytest.mark.parametrize("seq,ch", [(64, 2051), (16, 3), (1000, 64)])
def test_gdn2_scan(cuda, orc, seq, ch):
    r = np.random.default_rng(seq)
    g = r.uniform(0.5, 0.99, (seq, ch)).astype(np.float32)
    bg = r.uniform(0, 1, (seq, ch)).astype(np.float32)
    wg = r.uniform(0, 1, (seq, ch)).astype(np.float32)
    x = r.uniform(-1, 1, (seq, ch)).astype(np.float32)
    st = r.uniform(-1, 1, ch).astype(np.float32)
    s_want, st_want = orc.gdn2_scan(g, bg, wg, x, st)
    s = cuda.empty((seq, ch), dtype=cuda.float32, device="cuda")
    st_d = _t(cuda, st)
    ops.gdn2_gated_scan(_t(cuda, g), _t(cuda, bg), _t(cuda, wg), _t(cuda, x), s, st_d)
    if seq <= 128:
        assert np.array_equal(s.cpu().numpy(), s_want) and np.array_equal(st_d.cpu().numpy(), st_want)
    else:
        assert validate_pass(s.cpu().numpy(), s_want)


CONV = [(1, 2048), (2, 2048), (3, 2048), (4, 7), (5, 17), (16, 129), (33, 1), (64, 2051), (65, 8192),
        (512, 2048), (2048, 8192)]


@pytest.mark.parametrize("seq,ch", CONV)
def test_conv_bit_exact(cuda, orc, seq, ch):
    r = np.random.default_rng(seq * 7 + ch)
    x = r.uniform(-1, 1, (seq, ch)).astype(np.float32)
    w = r.uniform(-1, 1, (4, ch)).astype(np.float32)
    h = r.uniform(-1, 1, (3, ch)).astype(np.float32)
    o_want, h_want = orc.conv(x, w, h)
    out = cuda.empty((seq, ch), dtype=cuda.float32, device="cuda")
    h_d = _t(cuda, h)
    ops.causal_dwconv1d(_t(cuda, x), _t(cuda, w), out, h_d)
    assert np.array_equal(out.cpu().numpy(), o_want)
    assert np.array_equal(h_d.cpu().numpy(), h_want)


def test_conv_integer_exact_config0(cuda):
    """Config 0 full size, integer-valued x and w in {-3..3}: exact."""
    T, C = 2048, 8192
    r = np.random.default_rng(11)
    x = r.integers(-3, 4, (T, C)).astype(np.float32)
    w = r.integers(-3, 4, (4, C)).astype(np.float32)
    h = np.zeros((3, C), np.float32)
    out = cuda.empty((T, C), dtype=cuda.float32, device="cuda")
    ops.causal_dwconv1d(_t(cuda, x), _t(cuda, w), out, _t(cuda, h))
    full = np.concatenate([h, x]).astype(np.int64)
    want = sum(w[j].astype(np.int64) * full[j:j + T] for j in range(4))
    assert np.array_equal(out.cpu().numpy().astype(np.int64), want)


def test_conv_streaming_continuity_and_batch(cuda, orc):
    """Two calls with carried history == one call (test_gdn_sve.c streaming
    check), batched over sequences."""
    B, T, C = 2, 128, 2051
    r = np.random.default_rng(12)
    x = (r.uniform(0, 1, (B, T, C)) - 0.5).astype(np.float32)
    w = (r.uniform(0, 1, (4, C)) - 0.5).astype(np.float32)
    h = np.zeros((B, 3, C), np.float32)
    full = cuda.empty((B, T, C), dtype=cuda.float32, device="cuda")
    ops.causal_dwconv1d(_t(cuda, x), _t(cuda, w), full, _t(cuda, h))
    h_d = _t(cuda, h)
    a = cuda.empty((B, T // 2, C), dtype=cuda.float32, device="cuda")
    b = cuda.empty((B, T // 2, C), dtype=cuda.float32, device="cuda")
    ops.causal_dwconv1d(_t(cuda, x[:, :T // 2]), _t(cuda, w), a, h_d)
    ops.causal_dwconv1d(_t(cuda, x[:, T // 2:]), _t(cuda, w), b, h_d)
    assert cuda.equal(cuda.cat([a, b], 1), full)
    for i in range(B):
        o_want, h_want = orc.conv(x[i], w, h[i])
        assert np.array_equal(full[i].cpu().numpy(), o_want)
        assert np.array_equal(h_d[i].cpu().numpy(), h_want)


@pytest.mark.parametrize("kind", ["f16", "bf16"])
@pytest.mark.parametrize("seq,ch", [(64, 8192), (5, 17), (300, 64)])
def test_conv_narrow_io(cuda, orc, kind, seq, ch):
    r = np.random.default_rng(seq)
    xu = oracle.f32_to_u16(r.standard_normal((seq, ch)), kind)
    w = (r.standard_normal((4, ch)) * 0.5).astype(np.float32)
    hu = oracle.f32_to_u16(r.standard_normal((3, ch)), kind)
    o_want, h_want = orc.conv_narrow(xu, w, hu, kind)
    tdt = cuda.float16 if kind == "f16" else cuda.bfloat16
    xd = cuda.from_numpy(xu.view(np.int16).copy()).cuda().view(tdt)
    hd = cuda.from_numpy(hu.view(np.int16).copy()).cuda().view(tdt)
    out = cuda.empty((seq, ch), dtype=tdt, device="cuda")
    ops.causal_dwconv1d(xd, _t(cuda, w), out, hd)
    assert np.array_equal(out.view(cuda.int16).cpu().numpy().view(np.uint16), o_want)
    assert np.array_equal(hd.view(cuda.int16).cpu().numpy().view(np.uint16), h_want)


@pytest.mark.parametrize("M,K,N", [(1, 128, 128), (64, 128, 128), (1, 128, 2048), (64, 128, 2048),
                                   (1, 128, 130), (64, 128, 130), (1, 1024, 257), (3, 1, 5), (17, 33, 65)])
def test_matmul_bit_exact(cuda, orc, M, K, N):
    r = np.random.default_rng(M + K + N)
    A = r.uniform(-1, 1, (M, K)).astype(np.float32)
    B = r.uniform(-1, 1, (K, N)).astype(np.float32)
    Cm = cuda.empty((M, N), dtype=cuda.float32, device="cuda")
    ops.matmul(_t(cuda, A), _t(cuda, B), Cm)
    assert np.array_equal(Cm.cpu().numpy(), orc.matmul(A, B))


def test_matmul_k0_writes_zeros(cuda):
    Cm = cuda.full((2, 8), float("nan"), device="cuda")
    A = cuda.empty((2, 0), device="cuda")
    B = cuda.empty((0, 8), device="cuda")
    ops.matmul(A, B, Cm)
    assert cuda.count_nonzero(Cm).item() == 0
