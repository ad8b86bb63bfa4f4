"""GPU parity of the packed int8 matmul (kai_run_gdn_int8_pack_sm100a,
kai_run_gdn_matmul_int8_packed_sm100a): the reference's matmul_int8
(gdn_e2e_decode.c:608-681) over weights packed once for streaming -- the
weight stream for up to 16 activation rows, the row-tiled GEMM above.

Bars (written here):
  packing            bit-identical to a numpy restatement of the layout
                     (tiles of 256 columns, stages of 64 rows, [4][256][16]
                     signed codes per stage, 0 outside K x N)
  matmul             relative L2 <= 1e-5 against the oracle's k-ordered sums
                     (activations carried as 24-bit fixed point per row,
                     products summed exactly) and the reference test's bound
                     against the fp32 product (test_gdn_e2e_int8.c:79-161);
                     identical results from call to call
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2
from orionsbelt_b200 import ops

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _pack_np(q: np.ndarray) -> np.ndarray:
    K, N = q.shape
    tiles, S = -(-N // 256), -(-K // 64)
    full = np.zeros((S * 64, tiles * 256), np.int8)
    full[:K, :N] = q
    # [tile][stage][kg][c][i] = q[stage*64 + kg*16 + i][tile*256 + c]
    v = full.reshape(S, 4, 16, tiles, 256).transpose(3, 0, 1, 4, 2)
    return np.ascontiguousarray(v).reshape(-1)


def _quantized(orc, K, N, seed):
    r = np.random.default_rng(seed)
    B = r.uniform(-1, 1, (K, N)).astype(np.float32)
    B[:, 0] = 0.0
    return orc.quantize_int8(B), B


@pytest.mark.parametrize("K,N", [(64, 256), (66, 272), (2560, 528), (300, 48)])
def test_pack_layout_bit_identical(cuda, orc, K, N):
    (q_np, _), _ = _quantized(orc, K, N, K + N)
    qp = ops.pack_int8(cuda.from_numpy(q_np).cuda())
    assert np.array_equal(qp.cpu().numpy().view(np.int8), _pack_np(q_np))


SHAPES = [(64, 256), (66, 272), (300, 48), (2560, 9216), (9216, 2560), (4096, 2560), (2560, 2064)]


@pytest.mark.parametrize("M", [1, 2, 5, 15, 16, 17, 40, 64, 300])
@pytest.mark.parametrize("K,N", SHAPES)
def test_matmul_int8_packed_vs_oracle(cuda, orc, M, K, N):
    if M > 17 and K * N > 6_000_000:
        pytest.skip("several passes over large weights: covered by the 2560 x 2064 case")
    (q_np, s_np), B = _quantized(orc, K, N, 3 * K + N)
    A = np.random.default_rng(M * 1000 + K).uniform(-1, 1, (M, K)).astype(np.float32)
    want = orc.matmul_int8(A, q_np, s_np)
    qp = ops.pack_int8(cuda.from_numpy(q_np).cuda())
    s = cuda.from_numpy(s_np).cuda()
    Cm = cuda.full((M, N), float("nan"), device="cuda")
    ops.matmul_int8_packed(cuda.from_numpy(A).cuda(), qp, s, Cm)
    got = Cm.cpu().numpy()
    assert not np.isnan(got).any()
    assert rel_l2(got, want) < TOL, (M, K, N, rel_l2(got, want))
    c32 = A.astype(np.float64) @ B.astype(np.float64)
    bound = s_np.astype(np.float64)[None, :] * 0.5 * np.abs(A).sum(1, keepdims=True)
    assert (np.abs(got - c32) <= 2 * bound + 1e-6).all()


def test_matmul_int8_packed_lm_head_matches_row_major_path(cuda):
    """The config-4 LM head (2560 x 151936, 389 MB) at 16 rows: the packed
    path equals the row-major path (itself pinned to the oracle above)."""
    torch = cuda
    K, N, M = 2560, 151936, 16
    g = torch.Generator(device="cuda").manual_seed(7)
    W = torch.randn((K, N), device="cuda", generator=g) * 0.02
    q = torch.empty((K, N), dtype=torch.int8, device="cuda")
    s = torch.empty(N, device="cuda")
    ops.quantize_int8(W, q, s)
    del W
    A = torch.randn((M, K), device="cuda", generator=g)
    ref = torch.empty((M, N), device="cuda")
    ops.matmul_int8(A, q, s, ref)
    qp = ops.pack_int8(q)
    got = torch.full((M, N), float("nan"), device="cuda")
    ops.matmul_int8_packed(A, qp, s, got)
    assert not torch.isnan(got).any()
    assert rel_l2(got.cpu().numpy(), ref.cpu().numpy()) < TOL


def test_matmul_int8_packed_deterministic_and_repeated_shapes(cuda, orc):
    """Split tiles keep counters that each call resets: calls of different
    shapes in a row on one stream match the oracle, and a repeated call gives
    the same bits."""
    cases = [(16, 9216, 2560), (3, 4096, 1024), (16, 9216, 2560), (9, 8192, 512), (16, 2560, 4096)]
    first = {}
    for i, (M, K, N) in enumerate(cases):
        (q_np, s_np), _ = _quantized(orc, K, N, 50 + K + N)
        A = np.random.default_rng(K + N).uniform(-1, 1, (M, K)).astype(np.float32)
        qp = ops.pack_int8(cuda.from_numpy(q_np).cuda())
        s = cuda.from_numpy(s_np).cuda()
        Cm = cuda.full((M, N), float("nan"), device="cuda")
        ops.matmul_int8_packed(cuda.from_numpy(A).cuda(), qp, s, Cm)
        got = Cm.cpu().numpy()
        assert rel_l2(got, orc.matmul_int8(A, q_np, s_np)) < TOL, (i, M, K, N)
        if (M, K, N) in first:
            assert np.array_equal(first[(M, K, N)], got)
        first[(M, K, N)] = got


def test_matmul_int8_packed_rejects_unsupported_shapes(cuda):
    from orionsbelt_b200 import _lib

    assert _lib.lib().kai_gdn_int8_packed_bytes(64, 250) == 0  # N % 16
    assert _lib.lib().kai_gdn_int8_packed_bytes((1 << 17) + 4, 256) == 0  # K too long for int32 sums
    assert _lib.lib().kai_gdn_int8_packed_bytes(66, 256) == 2 * 16384  # ragged K: zero rows
    with pytest.raises(ValueError):
        ops.pack_int8(cuda.zeros((64, 250), dtype=cuda.int8, device="cuda"))
