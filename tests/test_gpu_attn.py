"""GPU parity of the GQA attention decode (gdn_e2e_decode.c:1532-1634
full_attn_real_forward, :1652-1830 full_attn_real_forward_int8kv; bf16 cache
as an extension) through kai_run_gdn_attention_decode_sm100a, against the
oracle (which is bit-identical to the reference's own functions).

Bars (written here):
  the appended cache entries   bit-identical to the oracle's
  outputs                      relative L2 <= 1e-5 (fp32 arithmetic in another
                               order: chunked softmax, fused multiply-add)
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2
from orionsbelt_b200 import ops

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _case(B, H, Hkv, D, max_ctx, kind, seed):
    r = np.random.default_rng(seed)
    q = r.uniform(-1, 1, (B, H, D)).astype(np.float32)
    kn, vn = (r.uniform(-1, 1, (B, Hkv, D)).astype(np.float32) for _ in range(2))
    ks = vs = None
    if kind == "f32":
        kc, vc = (r.uniform(-1, 1, (B, max_ctx, Hkv, D)).astype(np.float32) for _ in range(2))
    elif kind == "bf16":
        kc, vc = (r.integers(0, 1 << 16, (B, max_ctx, Hkv, D), dtype=np.uint32) for _ in range(2))
        # finite bf16 values of magnitude 2^-15 .. 2: sign, exponent 0x70-0x7f, any mantissa
        kc, vc = (((x & 0x807F) | (0x3800 + ((x >> 8) & 0x0F) * 0x80)).astype(np.uint16) for x in (kc, vc))
    else:
        kc, vc = (r.integers(-128, 128, (B, max_ctx, Hkv, D)).astype(np.int8) for _ in range(2))
        ks, vs = (r.uniform(0.002, 0.02, (B, Hkv)).astype(np.float32) for _ in range(2))
    return q, kn, vn, kc, vc, ks, vs


def _to_dev(cuda, a, kind):
    if kind == "bf16":
        return cuda.from_numpy(a.view(np.int16)).cuda().view(cuda.bfloat16)
    return cuda.from_numpy(np.ascontiguousarray(a)).cuda()


def _from_dev(cuda, t, kind):
    if kind == "bf16":
        return t.view(cuda.int16).cpu().numpy().view(np.uint16)
    return t.cpu().numpy()


def _run(cuda, q, kn, vn, kc, vc, ks, vs, pos, scale, kind):
    dev = [cuda.from_numpy(x).cuda() for x in (q, kn, vn)]
    kcd, vcd = _to_dev(cuda, kc, kind), _to_dev(cuda, vc, kind)
    o = cuda.full(q.shape, float("nan"), device="cuda")
    ksd = cuda.from_numpy(ks).cuda() if ks is not None else None
    vsd = cuda.from_numpy(vs).cuda() if vs is not None else None
    ops.attention_decode(*dev, kcd, vcd, o, pos, scale, ksd, vsd)
    return o.cpu().numpy(), _from_dev(cuda, kcd, kind), _from_dev(cuda, vcd, kind)


@pytest.mark.parametrize("kind", ["f32", "bf16", "i8"])
@pytest.mark.parametrize("B,H,Hkv,D,pos,max_ctx", [
    (1, 16, 4, 256, 0, 8), (1, 16, 4, 256, 63, 64), (1, 16, 4, 256, 64, 100), (1, 16, 4, 256, 1000, 1024),
    (2, 16, 4, 256, 4095, 4096), (3, 8, 8, 128, 200, 300), (2, 4, 2, 128, 511, 600), (1, 32, 4, 128, 777, 800),
    (1, 16, 4, 256, 32767, 32768),
    # 48-token tiles of the tensor-core kernel: one full tile, the first row of
    # the second, the last row of the second
    (1, 16, 4, 256, 47, 48), (1, 16, 4, 256, 48, 100), (2, 16, 4, 256, 95, 96),
])
def test_attention_decode_vs_oracle(cuda, orc, kind, B, H, Hkv, D, pos, max_ctx):
    if pos >= 32767 and kind != "bf16":
        pytest.skip("the long-context case runs once, with the bf16 cache")
    q, kn, vn, kc, vc, ks, vs = _case(B, H, Hkv, D, max_ctx, kind, pos + B * 7 + D)
    scale = 1.0 / np.sqrt(np.float32(D))
    o, kc_got, vc_got = _run(cuda, q, kn, vn, kc, vc, ks, vs, pos, scale, kind)
    o_want = orc.attn_decode(q, kn, vn, kc, vc, pos, scale, ks, vs)  # updates kc, vc in place
    assert np.array_equal(kc_got, kc) and np.array_equal(vc_got, vc)
    assert not np.isnan(o).any()
    assert rel_l2(o, o_want) < TOL, rel_l2(o, o_want)


@pytest.mark.parametrize("kind", ["f32", "bf16", "i8"])
def test_attention_decode_steps(cuda, orc, kind):
    """Eight decode steps in a row on one cache (the reference's ctx-sweep use:
    the cache grows by one token per call; for bf16 the new token moves through
    one tensor-core tile)."""
    B, H, Hkv, D, max_ctx = 1, 16, 4, 256, 600
    _, _, _, kc, vc, ks, vs = _case(B, H, Hkv, D, max_ctx, kind, 5)
    kcd, vcd = _to_dev(cuda, kc, kind), _to_dev(cuda, vc, kind)
    ksd = cuda.from_numpy(ks).cuda() if ks is not None else None
    vsd = cuda.from_numpy(vs).cuda() if vs is not None else None
    r = np.random.default_rng(9)
    for pos in range(500, 508):
        q = r.uniform(-1, 1, (B, H, D)).astype(np.float32)
        kn, vn = (r.uniform(-1, 1, (B, Hkv, D)).astype(np.float32) for _ in range(2))
        o = cuda.empty((B, H, D), device="cuda")
        ops.attention_decode(cuda.from_numpy(q).cuda(), cuda.from_numpy(kn).cuda(), cuda.from_numpy(vn).cuda(), kcd,
                             vcd, o, pos, 0.0625, ksd, vsd)
        o_want = orc.attn_decode(q, kn, vn, kc, vc, pos, 0.0625, ks, vs)
        assert rel_l2(o.cpu().numpy(), o_want) < TOL, pos
    assert np.array_equal(_from_dev(cuda, kcd, kind), kc) and np.array_equal(_from_dev(cuda, vcd, kind), vc)


def test_attention_decode_errors(cuda):
    from orionsbelt_b200 import _lib
    q = cuda.zeros((1, 6, 128), device="cuda")
    kn = cuda.zeros((1, 2, 128), device="cuda")
    kc = cuda.zeros((1, 16, 2, 128), device="cuda")
    o = cuda.empty((1, 6, 128), device="cuda")
    with pytest.raises(_lib.GdnError, match="per kv head"):
        ops.attention_decode(q, kn, kn, kc, kc.clone(), o, 3, 0.1)
    _lib.lib().kai_gdn_cuda_clear_error()
    q = cuda.zeros((1, 4, 128), device="cuda")
    with pytest.raises(_lib.GdnError, match="outside the cache"):
        ops.attention_decode(q, kn, kn, kc, kc.clone(), o[:, :4].contiguous(), 16, 0.1)
    _lib.lib().kai_gdn_cuda_clear_error()
