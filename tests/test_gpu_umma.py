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
