"""tcgen05 building blocks (orionsbelt_b200/csrc/umma.cuh) on the GPU.

A single-CTA GEMM through the self-test library writes A and B into shared
memory in the K-major / MN-major no-swizzle layouts, runs kind::f16 (bf16) or
kind::tf32 MMAs into TMEM and reads the accumulator back with the M=64 /
M=128 lane mapping.  Checked against numpy on the same rounded inputs.
"""
from __future__ import annotations

import ctypes as C
import itertools

import numpy as np
import pytest

import oracle
from conftest import rel_l2
from orionsbelt_b200 import build

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def selftest():
    lib = C.CDLL(str(build.SELFTEST_LIB))
    lib.umma_selftest_gemm.restype = C.c_int
    lib.umma_selftest_gemm.argtypes = [C.c_void_p] * 3 + [C.c_int] * 7 + [C.c_void_p]
    return lib


def _bf16(a):
    return oracle.u16_to_f32(oracle.f32_to_u16(a, "bf16"), "bf16")


CASES = [(M, N, K, a, b) for M, N, K in [(128, 64, 64), (128, 128, 128), (64, 64, 64), (64, 256, 64), (128, 256, 32)]
         for a, b in itertools.product([0, 1], [0, 1])]


@pytest.mark.parametrize("M,N,K,a_mn,b_mn", CASES)
def test_bf16_layouts(cuda, selftest, M, N, K, a_mn, b_mn):
    r = np.random.default_rng(M * 1000 + N + K + 10 * a_mn + b_mn)
    A = r.standard_normal((M, K)).astype(np.float32)
    B = r.standard_normal((K, N)).astype(np.float32)
    Ad, Bd = cuda.from_numpy(A).cuda(), cuda.from_numpy(B).cuda()
    D = cuda.full((M, N), float("nan"), device="cuda")
    err = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    rc = selftest.umma_selftest_gemm(Ad.data_ptr(), Bd.data_ptr(), D.data_ptr(), M, N, K, a_mn, b_mn, 0, 0,
                                     err.data_ptr())
    assert rc == 0 and err.item() == 0
    want = _bf16(A).astype(np.float64) @ _bf16(B).astype(np.float64)
    assert rel_l2(D.cpu().numpy(), want) < 1e-5


@pytest.mark.parametrize("M,N,K", [(128, 64, 64), (64, 128, 32)])
def test_tf32_kmajor(cuda, selftest, M, N, K):
    r = np.random.default_rng(M + N)
    A = r.standard_normal((M, K)).astype(np.float32)
    B = r.standard_normal((K, N)).astype(np.float32)
    Ad, Bd = cuda.from_numpy(A).cuda(), cuda.from_numpy(B).cuda()
    D = cuda.full((M, N), float("nan"), device="cuda")
    err = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    assert selftest.umma_selftest_gemm(Ad.data_ptr(), Bd.data_ptr(), D.data_ptr(), M, N, K, 0, 0, 1, 0,
                                       err.data_ptr()) == 0
    assert err.item() == 0
    assert rel_l2(D.cpu().numpy(), A.astype(np.float64) @ B.astype(np.float64)) < 3e-3


@pytest.mark.parametrize("N,b_mn", [(128, 1), (64, 0)])
def test_m64_upper_lane_half(cuda, selftest, N, b_mn):
    """An M=64 accumulator at TMEM lane offset 16 (the second of two
    interleaved half-quadrant tiles): rows 16w..16w+15 land in lanes
    32w+16..32w+31."""
    r = np.random.default_rng(N)
    A = r.standard_normal((64, 64)).astype(np.float32)
    B = r.standard_normal((64, N)).astype(np.float32)
    Ad, Bd = cuda.from_numpy(A).cuda(), cuda.from_numpy(B).cuda()
    D = cuda.full((64, N), float("nan"), device="cuda")
    err = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    assert selftest.umma_selftest_gemm(Ad.data_ptr(), Bd.data_ptr(), D.data_ptr(), 64, N, 64, 0, b_mn, 0, 1,
                                       err.data_ptr()) == 0
    assert err.item() == 0
    want = _bf16(A).astype(np.float64) @ _bf16(B).astype(np.float64)
    assert rel_l2(D.cpu().numpy(), want) < 1e-5


# ---------------------------------------------------------------- layout modes
# 0/1 K-/MN-major (k-groups / mn-groups inner), 2/3 the TMA-order variants,
# 5/6 K-/MN-major with the 128-byte swizzle, 4 = A operand in TMEM.
MODE_CASES = [
    (128, 64, 64, 2, 2), (128, 64, 128, 2, 3), (64, 64, 128, 2, 2), (128, 128, 64, 3, 3), (128, 64, 64, 3, 0),
    (128, 64, 128, 4, 2), (128, 128, 64, 4, 3), (128, 64, 64, 4, 0), (128, 128, 128, 4, 1),
    (128, 64, 128, 5, 5), (64, 64, 128, 5, 5), (128, 128, 64, 6, 6), (128, 64, 128, 6, 5), (128, 128, 64, 4, 6),
    (128, 64, 128, 4, 5),
]


@pytest.fixture(scope="module")
def selftest2(selftest):
    selftest.umma_selftest_gemm2.restype = C.c_int
    selftest.umma_selftest_gemm2.argtypes = [C.c_void_p] * 3 + [C.c_int] * 5 + [C.c_void_p]
    selftest.umma_selftest_tma.restype = C.c_int
    selftest.umma_selftest_tma.argtypes = [C.c_void_p, C.c_void_p] + [C.c_int] * 8 + [C.c_void_p]
    return selftest


@pytest.mark.parametrize("M,N,K,a_mode,b_mode", MODE_CASES)
def test_layout_modes(cuda, selftest2, M, N, K, a_mode, b_mode):
    r = np.random.default_rng(7 * M + 3 * N + K + 100 * a_mode + 10 * b_mode)
    A = r.standard_normal((M, K)).astype(np.float32)
    B = r.standard_normal((K, N)).astype(np.float32)
    Ad, Bd = cuda.from_numpy(A).cuda(), cuda.from_numpy(B).cuda()
    D = cuda.full((M, N), float("nan"), device="cuda")
    err = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    rc = selftest2.umma_selftest_gemm2(Ad.data_ptr(), Bd.data_ptr(), D.data_ptr(), M, N, K, a_mode, b_mode,
                                       err.data_ptr())
    assert rc == 0 and err.item() == 0
    want = _bf16(A).astype(np.float64) @ _bf16(B).astype(np.float64)
    got = D.cpu().numpy()
    if M == 64:
        got = got[:64]
    assert rel_l2(got, want) < 1e-5


def _tile_expected(x, b, t0, h, swz):
    """Byte layout the TMA chunk load should produce (uint16 view, 8192 entries)."""
    T = x.shape[1]
    out = np.zeros(8192, np.uint16)
    for t in range(64):
        for d in range(128):
            v = x[b, t0 + t, h, d] if t0 + t < T else 0
            if not swz:
                off = (d // 8) * 1024 + (t // 8) * 128 + (t % 8) * 16 + (d % 8) * 2
            else:
                chunk = (d % 64) // 8
                off = (d // 64) * 8192 + t * 128 + ((chunk ^ (t % 8)) * 16) + (d % 8) * 2
            out[off // 2] = v
    return out


@pytest.mark.parametrize("swz", [0, 1])
@pytest.mark.parametrize("t0", [0, 64, 100])
def test_tma_chunk_tile(cuda, selftest2, swz, t0):
    B, T, H = 2, 130, 3
    r = np.random.default_rng(5)
    x = r.integers(1, 60000, size=(B, T, H, 128), dtype=np.uint16)
    src = cuda.from_numpy(x.view(np.int16)).cuda()
    out = cuda.zeros(8192, dtype=cuda.int16, device="cuda")
    err = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    rc = selftest2.umma_selftest_tma(src.data_ptr(), out.data_ptr(), 1, B, T, H, t0, 2, 1, swz, err.data_ptr())
    assert rc == 0 and err.item() == 0
    got = out.cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(got, _tile_expected(x, 1, t0, 2, swz))


def test_bounded_wait_runs_out(cuda, selftest):
    """A wait on an mbarrier that nothing completes gives up after its poll
    limit, records the timeout in the error word and lets the kernel finish
    (the pattern every wait of the chunk scan uses)."""
    selftest.umma_selftest_timeout.restype = C.c_int
    selftest.umma_selftest_timeout.argtypes = [C.c_void_p, C.c_void_p]
    err = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    done = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    assert selftest.umma_selftest_timeout(err.data_ptr(), done.data_ptr()) == 0
    assert err.item() == 1 and done.item() == 1
