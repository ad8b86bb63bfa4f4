"""GPU parity of the causal prompt attention (kai_run_gdn_attention_prefill_sm100a)
against the oracle's attention decode (bit-identical to the reference's
full_attn_real_forward, gdn_e2e_decode.c:1532-1634, over a bf16 cache) called
once per prompt position, as the reference feeds a prompt.

Bar (written here): relative L2 <= 1e-4 over all outputs and 1e-3 per query
row for scores of order one (queries and softmax weights carry two bf16
terms, 16 significant bits; products summed in fp32 in another order); for
scores rising to ~60 (the case that raises the running maximum many times)
the score error grows with the score, |s| 2^-17, and the bar is 1e-3.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2
from orionsbelt_b200 import ops

pytestmark = pytest.mark.gpu

TOL = 1e-4


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    import oracle

    return oracle.f32_to_u16(np.ascontiguousarray(x, np.float32), "bf16")


def _bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def _reference(orc, q, kc, vc, pos0, scale):
    """o[b][t] = the oracle's decode of query t at position pos0 + t."""
    B, T, H, D = q.shape
    out = np.empty_like(q)
    k2, v2 = kc.copy(), vc.copy()
    for t in range(T):
        pos = pos0 + t
        kn, vn = _bits_to_f32(kc[:, pos]), _bits_to_f32(vc[:, pos])  # re-appending the cached values
        out[:, t] = orc.attn_decode(q[:, t], kn, vn, k2, v2, pos, scale)
    return out


CASES = [
    # B, T, pos0, H, Hkv, D, query scale, growing keys
    (2, 200, 0, 16, 4, 256, 1.0, False),
    (1, 150, 37, 16, 4, 256, 1.0, False),
    (1, 64, 0, 16, 4, 256, 1.0, False),
    (1, 1, 300, 16, 4, 256, 1.0, False),
    (1, 130, 0, 8, 8, 128, 1.0, False),
    (1, 100, 5, 16, 2, 128, 1.0, False),
    (1, 90, 0, 4, 2, 256, 1.0, False),
    (1, 260, 0, 16, 4, 256, 1.0, True),  # rising scores (to ~60): the running maximum is raised many times
]


@pytest.mark.parametrize("B,T,pos0,H,Hkv,D,qs,grow", CASES)
def test_attention_prefill_vs_oracle(cuda, orc, B, T, pos0, H, Hkv, D, qs, grow):
    torch = cuda
    r = np.random.default_rng(T * 7 + pos0 + D)
    max_ctx = pos0 + T + 17
    q = (r.uniform(-1, 1, (B, T, H, D)) * qs).astype(np.float32)
    kf = r.uniform(-1, 1, (B, max_ctx, Hkv, D)).astype(np.float32)
    if grow:
        kf = np.abs(kf) * (1.0 + np.arange(max_ctx)[None, :, None, None] / 20.0)
        q = np.abs(q)
    kc, vc = _bf16_bits(kf), _bf16_bits(r.uniform(-1, 1, (B, max_ctx, Hkv, D)))
    scale = 1.0 / np.sqrt(D)
    want = _reference(orc, q, kc, vc, pos0, scale)
    kd = torch.from_numpy(kc.view(np.int16)).cuda().view(torch.bfloat16)
    vd = torch.from_numpy(vc.view(np.int16)).cuda().view(torch.bfloat16)
    o = torch.full((B, T, H, D), float("nan"), device="cuda")
    ops.attention_prefill(torch.from_numpy(q).cuda(), kd, vd, o, pos0, scale)
    got = o.cpu().numpy()
    assert not np.isnan(got).any()
    tol = 10 * TOL if grow else TOL
    assert rel_l2(got, want) < tol, rel_l2(got, want)
    rows = np.sqrt(((got - want) ** 2).sum(-1) / np.maximum((want**2).sum(-1), 1e-30))
    assert rows.max() < 10 * tol, rows.max()
    # the caches are read only
    assert np.array_equal(kd.view(torch.int16).cpu().numpy().view(np.uint16), kc)


def test_attention_prefill_rejects_bad_arguments(cuda):
    from orionsbelt_b200 import _lib

    torch = cuda
    q = torch.zeros((1, 4, 6, 128), device="cuda")
    kc = torch.zeros((1, 8, 2, 128), dtype=torch.bfloat16, device="cuda")
    o = torch.zeros_like(q)
    with pytest.raises(_lib.GdnError):  # 3 query heads per kv head
        ops.attention_prefill(q, kc, kc, o, 0, 0.1)
    q = torch.zeros((1, 4, 4, 128), device="cuda")
    o = torch.zeros_like(q)
    with pytest.raises(_lib.GdnError):  # positions past the cache
        ops.attention_prefill(q, kc, kc, o, 6, 0.1)
