"""The C ABI surface of libkai_gdn_cuda.so (CPU only: no compute calls).

* The library loads and exports every symbol include/kai_gdn_cuda.h declares,
  and the Python binding declares exactly that set.
* The drop-in symbols keep the reference's exact signatures
  (kleidiai_submission/kai/ukernels/gdn/*.h, gdn_sve.h, gdn_delta_matmul.h).
* Host-side argument checks answer without touching a GPU: zero-size drop-in
  calls are no-ops, device entry points reject bad arguments with a status and
  a message, and nothing aborts the process.
"""
from __future__ import annotations

import ctypes as C
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

from orionsbelt_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "kai_gdn_cuda.h"


def header_symbols() -> set[str]:
    text = "\n".join(ln for ln in HEADER.read_text().splitlines() if not ln.startswith("#"))
    return set(re.findall(r"KAI_GDN_API\s+(?:const\s+)?\w+\s*\*?\s*(\w+)\s*\(", text))


def test_header_and_binding_agree():
    assert header_symbols() == set(_lib.SIGNATURES), header_symbols() ^ set(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    missing = header_symbols() - exported
    assert not missing, missing


def test_library_loads_and_binds(lib):
    assert lib.kai_gdn_cuda_version().startswith(b"kai_gdn_cuda")


def test_no_cuda_runtime_dependency_on_host_paths():
    """The CUDA runtime is linked statically: the library needs no libcudart."""
    out = subprocess.run(["ldd", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    assert "libcudart" not in out


def test_dropin_signatures_match_reference_headers():
    """Compile a C file that includes our header and re-declares the reference
    prototypes (text of kai_gdn_*.h / gdn_sve.h / gdn_delta_matmul.h with
    __fp16 as uint16_t): conflicting types would be a compile error."""
    protos = """
    void kai_run_gdn_cumdecay_f32_sve(const float *a, float *decay, size_t seq, size_t channels);
    void kai_run_gdn_gated_scan_f32_sve(const float *g, const float *x, float *s, float *state, size_t seq, size_t channels);
    void kai_run_gdn_causal_dwconv1d_f32_k4_sve(const float *in, const float *w, float *out, float *hist, size_t seq, size_t channels);
    void kai_run_gdn_gemv_f32_f32_f32_1x4_neon(const float *a, const float *b, float *c, size_t k, size_t n);
    void gdn_cumdecay_f32(const float *restrict a, float *restrict decay, size_t seq, size_t channels);
    void gdn_gated_scan_f32(const float *restrict g, const float *restrict x, float *restrict s, float *restrict state, size_t seq, size_t channels);
    void gdn_causal_dwconv1d_f32(const float *restrict in, const float *restrict w, float *restrict out, float *restrict hist, size_t seq, size_t channels);
    void gdn_cumdecay_f16(const float *restrict a, uint16_t *restrict decay, size_t seq, size_t channels);
    void gdn_gated_scan_f16(const float *restrict g, const float *restrict x, float *restrict s, uint16_t *restrict state, size_t seq, size_t channels);
    void gdn_cumdecay_bf16(const float *restrict a, uint16_t *restrict decay, size_t seq, size_t channels);
    void gdn_gated_scan_bf16(const float *restrict g, const float *restrict x, float *restrict s, uint16_t *restrict state, size_t seq, size_t channels);
    void gdn2_gated_scan_f32(const float *restrict g, const float *restrict b_gate, const float *restrict w_gate, const float *restrict x, float *restrict s, float *restrict state, size_t seq, size_t channels);
    void gdn_delta_rule_matmul(const float *restrict A, const float *restrict B, float *restrict C, size_t M, size_t K, size_t N);
    """
    src = f'#include "kai_gdn_cuda.h"\n{protos}\nint main(void){{return 0;}}\n'
    tmp = Path(subprocess.run(["mktemp", "-d"], capture_output=True, text=True).stdout.strip())
    (tmp / "t.c").write_text(src)
    r = subprocess.run(["gcc", "-std=c11", "-Werror", "-c", "-I", str(ROOT / "include"), str(tmp / "t.c"),
                        "-o", str(tmp / "t.o")], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_zero_size_dropin_calls_are_noops(lib):
    """seq == 0 / channels == 0 touch nothing (test_kai_gdn.c:520-637), and
    return before any CUDA call, so they work without a GPU."""
    got = np.array([42.0], np.float32)
    lib.kai_run_gdn_cumdecay_f32_sve(got.ctypes.data, got.ctypes.data, 0, 8)
    lib.kai_run_gdn_cumdecay_f32_sve(got.ctypes.data, got.ctypes.data, 8, 0)
    st = np.array([1.0, -2.0, 3.0, -4.0], np.float32)
    lib.kai_run_gdn_gated_scan_f32_sve(got.ctypes.data, got.ctypes.data, got.ctypes.data, st.ctypes.data, 0, 4)
    hist = np.arange(6, dtype=np.float32)
    lib.kai_run_gdn_causal_dwconv1d_f32_k4_sve(got.ctypes.data, got.ctypes.data, got.ctypes.data,
                                               hist.ctypes.data, 0, 2)
    lib.kai_run_gdn_gemv_f32_f32_f32_1x4_neon(got.ctypes.data, got.ctypes.data, got.ctypes.data, 4, 0)
    assert got[0] == 42.0
    assert np.array_equal(st, [1.0, -2.0, 3.0, -4.0])
    assert np.array_equal(hist, np.arange(6, dtype=np.float32))
    assert lib.kai_gdn_cuda_last_status() == _lib.OK


def test_device_entry_points_reject_bad_arguments(lib):
    lib.kai_gdn_cuda_clear_error()
    assert lib.kai_run_gdn_delta_rule_decode_sm100a(None, None) == _lib.ERR_INVALID
    assert b"null" in lib.kai_gdn_cuda_last_error()
    args = _lib.DecodeArgs()
    args.batch, args.heads_k, args.heads_v, args.dk, args.dv = 1, 3, 4, 128, 128
    args.state = args.q = args.k = args.v = args.g = args.beta = args.o = 256
    assert lib.kai_run_gdn_delta_rule_decode_sm100a(C.byref(args), None) == _lib.ERR_INVALID
    assert b"multiple" in lib.kai_gdn_cuda_last_error()
    c = _lib.ChunkArgs()
    c.batch, c.seq, c.heads_k, c.heads_v, c.dk, c.dv, c.chunk = 1, 8, 1, 1, 128, 128, 32
    c.q = c.k = c.v = c.g = c.beta = c.state = c.o = 256
    assert lib.kai_run_gdn_chunk_delta_rule_sm100a(C.byref(c), None) == _lib.ERR_UNSUPPORTED
    assert lib.kai_run_gdn_cumdecay_sm100a(None, None, 0, 1, 4, 4, None) == _lib.ERR_INVALID
    assert lib.kai_run_gdn_cumdecay_sm100a(None, None, 0, 0, 4, 4, None) == _lib.OK  # empty: no-op
    assert lib.kai_run_gdn_causal_dwconv1d_k4_sm100a(256, 256, 256, 256, 9, 1, 4, 4, None) == _lib.ERR_INVALID
    lib.kai_gdn_cuda_clear_error()
    assert lib.kai_gdn_cuda_last_status() == _lib.OK and lib.kai_gdn_cuda_last_error() == b""


def test_python_layer_fails_loudly_without_library(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "missing.so")
    with pytest.raises(ImportError):
        _lib.lib()


def test_oracle_library_loads(orc):
    assert orc.num_threads() >= 1
