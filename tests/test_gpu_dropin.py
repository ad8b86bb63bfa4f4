"""The drop-in claim, on the GPU.

1. The reference's OWN C test programs (kleidiai_submission/test_kai_gdn.c and
   src/orionsbelt/engines/cpu/kernels/test_gdn_{sve,mixed,delta_matmul}.c),
   compiled from the reference sources by oracle/Makefile and linked against
   libkai_gdn_cuda.so instead of the reference kernels, pass unchanged --
   including test_gdn_sve.c's bit-identity gates.
2. The drop-in symbols, called with host pointers through ctypes, are
   bit-identical to the reference build (oracle/_ref/libgdnref.so).
"""
from __future__ import annotations

import subprocess
from pathlib import Path

import numpy as np
import pytest

import oracle
from orionsbelt_b200 import ops

pytestmark = pytest.mark.gpu

REF_DIR = Path(oracle.__file__).resolve().parent / "_ref"
PROGRAMS = ["test_kai_gdn_cuda", "test_gdn_sve_cuda", "test_gdn_mixed_cuda", "test_gdn_delta_matmul_cuda"]


@pytest.mark.parametrize("prog", PROGRAMS)
def test_reference_test_program_passes_against_cuda_library(cuda, prog):
    exe = REF_DIR / prog
    if not exe.exists():
        pytest.skip(f"{exe} not built (needs the reference tree at build time)")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-3000:]
    if prog == "test_kai_gdn_cuda":
        assert "ALL TESTS PASSED" in out
    if prog == "test_gdn_sve_cuda":
        assert "gated_scan bit-identical to matched reference: YES" in out
        assert "cumdecay bit-identical to matched reference: YES" in out
        assert "conv streaming bit-identical: YES" in out


def _need_ref(ref):
    if ref is None:
        pytest.skip("oracle/_ref/libgdnref.so not built")


@pytest.mark.parametrize("seq,ch", [(64, 2560), (1, 4096), (17, 33)])
def test_host_pointer_dropin_bit_identical(cuda, ref, seq, ch):
    _need_ref(ref)
    r = np.random.default_rng(seq + ch)
    a = r.uniform(0.5, 1.5, (seq, ch)).astype(np.float32)
    d = np.empty_like(a)
    ops.kai_run_gdn_cumdecay_f32_sve(a, d)
    assert np.array_equal(d, ref.kai_cumdecay(a))
    g = r.uniform(-0.99, 0.99, (seq, ch)).astype(np.float32)
    x = r.uniform(-2, 2, (seq, ch)).astype(np.float32)
    st = r.uniform(-1, 1, ch).astype(np.float32)
    s = np.empty_like(x)
    st_got = st.copy()
    ops.kai_run_gdn_gated_scan_f32_sve(g, x, s, st_got)
    s_want, st_want = ref.gated_scan(g, x, st)
    assert np.array_equal(s, s_want) and np.array_equal(st_got, st_want)
    w = r.uniform(-1, 1, (4, ch)).astype(np.float32)
    h = r.uniform(-1, 1, (3, ch)).astype(np.float32)
    o = np.empty_like(x)
    h_got = h.copy()
    ops.kai_run_gdn_causal_dwconv1d_f32_k4_sve(x, w, o, h_got)
    o_want, h_want = ref.conv(x, w, h)
    assert np.array_equal(o, o_want) and np.array_equal(h_got, h_want)
    for kind in ("f16", "bf16"):
        dn = np.empty((seq, ch), np.uint16)
        ops.gdn_cumdecay_narrow(a, dn, kind)
        assert np.array_equal(dn, ref.cumdecay_narrow(a, kind))
        stn = oracle.f32_to_u16(st, kind)
        stn_got = stn.copy()
        ops.gdn_gated_scan_narrow(g, x, s, stn_got, kind)
        s_want, stn_want = ref.gated_scan_narrow(g, x, stn, kind)
        assert np.array_equal(s, s_want) and np.array_equal(stn_got, stn_want)


def test_host_pointer_gemv_and_matmul_bit_identical(cuda, ref):
    _need_ref(ref)
    r = np.random.default_rng(2)
    A = r.uniform(-1, 1, (64, 128)).astype(np.float32)
    B = r.uniform(-1, 1, (128, 2048)).astype(np.float32)
    Cm = np.empty((64, 2048), np.float32)
    ops.gdn_delta_rule_matmul(A, B, Cm)
    assert np.array_equal(Cm, ref.matmul(A, B))
    c = np.empty(2048, np.float32)
    ops.kai_run_gdn_gemv_f32_f32_f32_1x4_neon(A[0].copy(), B, c)
    assert np.array_equal(c, ref.gemv(A[0], B))


def test_dropin_accepts_device_pointers(cuda, ref):
    """Device pointers are used in place (no staging)."""
    _need_ref(ref)
    from orionsbelt_b200._lib import lib
    a = np.random.default_rng(3).uniform(0.5, 1.5, (64, 100)).astype(np.float32)
    ad = cuda.from_numpy(a).cuda()
    dd = cuda.empty_like(ad)
    lib().kai_run_gdn_cumdecay_f32_sve(ad.data_ptr(), dd.data_ptr(), 64, 100)
    assert lib().kai_gdn_cuda_last_status() == 0
    assert np.array_equal(dd.cpu().numpy(), ref.kai_cumdecay(a))
