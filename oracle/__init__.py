"""Parity oracle for the GDN hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
``--impl reference`` legs may import this package.  The product library
(orionsbelt_b200/libkai_gdn_cuda.so) never calls into it and has no CPU
fallback.

Two CPU implementations are exposed through ctypes:

* ``orc``: liboracle.so, built from gdn_oracle.c -- a restatement of the
  reference's arithmetic (file:line citations in that file), bit-identical to
  the reference's scalar path where the reference has code, plus the token-loop
  and chunked-WY forms of the matrix-state delta rule.
* ``ref``: _ref/libgdnref.so, the reference's OWN C kernels compiled from
  source by oracle/Makefile (absent when the reference tree was not available
  at build time; then ``ref`` is None).

Arrays are numpy, C-contiguous; the wrappers allocate outputs and copy in/out
buffers so callers keep their inputs.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libgdnref.so"
INT8_REF_SO = HERE / "_ref" / "libint8ref.so"
ATTN_REF_SO = HERE / "_ref" / "libattnref.so"
E2E_REF_SO = HERE / "_ref" / "libe2eref.so"
ATTN_I8_REF_SO = HERE / "_ref" / "libattnref_i8.so"

_f = C.POINTER(C.c_float)
_u16 = C.POINTER(C.c_uint16)
_sz = C.c_size_t


def reference_root():
    """The reference source tree, from the ORIONSBELT_REF environment variable
    (None when it is unset or not a directory)."""
    r = os.environ.get("ORIONSBELT_REF")
    return Path(r) if r and Path(r).is_dir() else None


def build(ref: bool = True) -> None:
    """Compile liboracle.so (and, when ORIONSBELT_REF names the reference tree, _ref/)."""
    subprocess.run(["make", "-s", "-C", str(HERE), "oracle"], check=True)
    if ref and reference_root() is not None:
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", "ref-tests"], check=True)


def _load(path: Path):
    if not path.exists():
        return None
    return C.CDLL(str(path))


def _p(a: np.ndarray, dtype) -> C.POINTER:
    assert a.flags["C_CONTIGUOUS"] and a.dtype == dtype, (a.dtype, dtype)
    if dtype == np.int8:
        return a.ctypes.data_as(C.POINTER(C.c_int8))
    return a.ctypes.data_as(_f if dtype == np.float32 else _u16)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


class _Kernels:
    """The four kai ops and the gdn_sve.h twins, on one of the two libraries."""

    def __init__(self, lib, prefix: str):
        self.lib = lib
        self.prefix = prefix

    def _fn(self, name):
        return getattr(self.lib, self.prefix + name)

    def cumdecay(self, a):
        a = _f32(a)
        out = np.empty_like(a)
        self._fn("cumdecay_f32")(_p(a, np.float32), _p(out, np.float32), _sz(a.shape[0]), _sz(a.shape[1]))
        return out

    def cumdecay_narrow(self, a, kind: str):
        a = _f32(a)
        out = np.empty(a.shape, np.uint16)
        self._fn("cumdecay_" + kind)(_p(a, np.float32), _p(out, np.uint16), _sz(a.shape[0]), _sz(a.shape[1]))
        return out

    def gated_scan(self, g, x, state):
        g, x = _f32(g), _f32(x)
        st = _f32(state).copy()
        s = np.empty_like(x)
        self._fn("gated_scan_f32")(_p(g, np.float32), _p(x, np.float32), _p(s, np.float32),
                                   _p(st, np.float32), _sz(x.shape[0]), _sz(x.shape[1]))
        return s, st

    def gated_scan_narrow(self, g, x, state_u16, kind: str):
        g, x = _f32(g), _f32(x)
        st = np.ascontiguousarray(state_u16, dtype=np.uint16).copy()
        s = np.empty_like(x)
        self._fn("gated_scan_" + kind)(_p(g, np.float32), _p(x, np.float32), _p(s, np.float32),
                                       _p(st, np.uint16), _sz(x.shape[0]), _sz(x.shape[1]))
        return s, st

    def conv(self, x, w, hist):
        x, w = _f32(x), _f32(w)
        h = _f32(hist).copy()
        out = np.empty_like(x)
        self._fn("causal_dwconv1d_f32")(_p(x, np.float32), _p(w, np.float32), _p(out, np.float32),
                                        _p(h, np.float32), _sz(x.shape[0]), _sz(x.shape[1]))
        return out, h


class _Ref(_Kernels):
    """The reference's own build: kai_run_* and gdn_* symbols."""

    def __init__(self, lib):
        super().__init__(lib, "gdn_")

    def kai_cumdecay(self, a):
        a = _f32(a)
        out = np.empty_like(a)
        self.lib.kai_run_gdn_cumdecay_f32_sve(_p(a, np.float32), _p(out, np.float32), _sz(a.shape[0]),
                                              _sz(a.shape[1]))
        return out

    def matmul(self, A, B):
        A, B = _f32(A), _f32(B)
        Cm = np.empty((A.shape[0], B.shape[1]), np.float32)
        self.lib.gdn_delta_rule_matmul(_p(A, np.float32), _p(B, np.float32), _p(Cm, np.float32),
                                       _sz(A.shape[0]), _sz(A.shape[1]), _sz(B.shape[1]))
        return Cm

    def gemv(self, a, b):
        a, b = _f32(a), _f32(b)
        c = np.empty((b.shape[1],), np.float32)
        self.lib.kai_run_gdn_gemv_f32_f32_f32_1x4_neon(_p(a, np.float32), _p(b, np.float32), _p(c, np.float32),
                                                       _sz(b.shape[0]), _sz(b.shape[1]))
        return c

    def gdn2_scan(self, g, bg, wg, x, state):
        g, bg, wg, x = map(_f32, (g, bg, wg, x))
        st = _f32(state).copy()
        s = np.empty_like(x)
        self.lib.gdn2_gated_scan_f32(_p(g, np.float32), _p(bg, np.float32), _p(wg, np.float32),
                                     _p(x, np.float32), _p(s, np.float32), _p(st, np.float32),
                                     _sz(x.shape[0]), _sz(x.shape[1]))
        return s, st


class _Oracle(_Kernels):
    """The restatement in gdn_oracle.c."""

    def __init__(self, lib):
        super().__init__(lib, "orc_")
        lib.orc_num_threads.restype = C.c_int

    def cumsum(self, g):
        g = _f32(g)
        out = np.empty_like(g)
        self.lib.orc_cumsum_f32(_p(g, np.float32), _p(out, np.float32), _sz(g.shape[0]), _sz(g.shape[1]))
        return out

    def matmul(self, A, B):
        A, B = _f32(A), _f32(B)
        Cm = np.empty((A.shape[0], B.shape[1]), np.float32)
        self.lib.orc_matmul_f32(_p(A, np.float32), _p(B, np.float32), _p(Cm, np.float32),
                                _sz(A.shape[0]), _sz(A.shape[1]), _sz(B.shape[1]))
        return Cm

    def gemv(self, a, b):
        return self.matmul(np.asarray(a, np.float32)[None, :], b)[0]

    def gdn2_scan(self, g, bg, wg, x, state):
        g, bg, wg, x = map(_f32, (g, bg, wg, x))
        st = _f32(state).copy()
        s = np.empty_like(x)
        self.lib.orc_gdn2_gated_scan_f32(_p(g, np.float32), _p(bg, np.float32), _p(wg, np.float32),
                                         _p(x, np.float32), _p(s, np.float32), _p(st, np.float32),
                                         _sz(x.shape[0]), _sz(x.shape[1]))
        return s, st

    def conv_narrow(self, x_u16, w, hist_u16, kind: str):
        x = np.ascontiguousarray(x_u16, dtype=np.uint16)
        w = _f32(w)
        h = np.ascontiguousarray(hist_u16, dtype=np.uint16).copy()
        out = np.empty_like(x)
        self.lib.orc_causal_dwconv1d_narrow(_p(x, np.uint16), _p(w, np.float32), _p(out, np.uint16),
                                            _p(h, np.uint16), _sz(x.shape[0]), _sz(x.shape[1]),
                                            C.c_int(1 if kind == "bf16" else 0))
        return out, h

    def delta_rule_step(self, S, k, v, q, beta, decay):
        """One head, one token: gpu/gdn_gpu_validate.c:100-118 (scale 1)."""
        S = _f32(S).copy()
        k, v, q = map(_f32, (k, v, q))
        out = np.empty((S.shape[1],), np.float32)
        self.lib.orc_delta_rule_step(_p(S, np.float32), _p(k, np.float32), _p(v, np.float32),
                                     _p(q, np.float32), C.c_float(beta), C.c_float(decay),
                                     _p(out, np.float32), _sz(S.shape[0]), _sz(S.shape[1]))
        return S, out

    def delta_rule_decode(self, S, q, k, v, g, beta, scale=1.0, nthreads=0, copy=True):
        """S [B][Hv][dk][dv], q,k [B][Hk][dk], v [B][Hv][dv], g,beta [B][Hv].
        copy=False updates S (float32, C-contiguous) in place."""
        if copy:
            S = _f32(S).copy()
        else:
            assert S.dtype == np.float32 and S.flags["C_CONTIGUOUS"]
        q, k, v, g, beta = map(_f32, (q, k, v, g, beta))
        B, Hv, dk, dv = S.shape
        Hk = q.shape[1]
        o = np.empty((B, Hv, dv), np.float32)
        self.lib.orc_delta_rule_decode(_p(S, np.float32), _p(q, np.float32), _p(k, np.float32),
                                       _p(v, np.float32), _p(g, np.float32), _p(beta, np.float32),
                                       _p(o, np.float32), _sz(B), _sz(Hk), _sz(Hv), _sz(dk), _sz(dv),
                                       C.c_float(scale), C.c_int(nthreads))
        return S, o

    def delta_rule_seq(self, S, q, k, v, g, beta, scale=1.0, nthreads=0):
        """Token loop.  q,k [B][T][Hk][dk], v [B][T][Hv][dv], g,beta [B][T][Hv]."""
        S = _f32(S).copy()
        q, k, v, g, beta = map(_f32, (q, k, v, g, beta))
        B, T, Hk, dk = q.shape
        Hv, dv = v.shape[2], v.shape[3]
        o = np.empty((B, T, Hv, dv), np.float32)
        self.lib.orc_delta_rule_seq(_p(S, np.float32), _p(q, np.float32), _p(k, np.float32),
                                    _p(v, np.float32), _p(g, np.float32), _p(beta, np.float32),
                                    _p(o, np.float32), _sz(B), _sz(T), _sz(Hk), _sz(Hv), _sz(dk), _sz(dv),
                                    C.c_float(scale), C.c_int(nthreads))
        return S, o

    def gdn2_decode(self, S, q, k, v, g, bgate, wgate, scale=1.0, nthreads=0):
        """GDN-2 step.  S [B][Hv][dk][dv], q,k [B][Hk][dk], v,wgate [B][Hv][dv], g,bgate [B][Hv][dk]."""
        S = _f32(S).copy()
        q, k, v, g, bgate, wgate = map(_f32, (q, k, v, g, bgate, wgate))
        B, Hv, dk, dv = S.shape
        Hk = q.shape[1]
        o = np.empty((B, Hv, dv), np.float32)
        self.lib.orc_gdn2_decode(_p(S, np.float32), _p(q, np.float32), _p(k, np.float32), _p(v, np.float32),
                                 _p(g, np.float32), _p(bgate, np.float32), _p(wgate, np.float32),
                                 _p(o, np.float32), _sz(B), _sz(Hk), _sz(Hv), _sz(dk), _sz(dv),
                                 C.c_float(scale), C.c_int(nthreads))
        return S, o

    def gdn2_seq(self, S, q, k, v, g, bgate, wgate, scale=1.0, nthreads=0):
        """GDN-2 token loop.  q,k [B][T][Hk][dk], v,wgate [B][T][Hv][dv], g,bgate [B][T][Hv][dk]."""
        S = _f32(S).copy()
        q, k, v, g, bgate, wgate = map(_f32, (q, k, v, g, bgate, wgate))
        B, T, Hk, dk = q.shape
        Hv, dv = v.shape[2], v.shape[3]
        o = np.empty((B, T, Hv, dv), np.float32)
        self.lib.orc_gdn2_seq(_p(S, np.float32), _p(q, np.float32), _p(k, np.float32), _p(v, np.float32),
                              _p(g, np.float32), _p(bgate, np.float32), _p(wgate, np.float32),
                              _p(o, np.float32), _sz(B), _sz(T), _sz(Hk), _sz(Hv), _sz(dk), _sz(dv),
                              C.c_float(scale), C.c_int(nthreads))
        return S, o

    def quantize_int8(self, B):
        """B [K][N] fp32 -> (q [K][N] int8, s [N] fp32): gdn_e2e_decode.c:175-199."""
        B = _f32(B)
        K, N = B.shape
        q = np.empty((K, N), np.int8)
        s = np.empty((N,), np.float32)
        self.lib.orc_quantize_int8(_p(B, np.float32), _p(q, np.int8), _p(s, np.float32), _sz(K), _sz(N))
        return q, s

    def matmul_int8(self, A, q, s, nthreads=0):
        """A [M][K] fp32, q [K][N] int8, s [N] -> C [M][N] (k-ordered sums, then * s)."""
        A, s = _f32(A), _f32(s)
        q = np.ascontiguousarray(q, dtype=np.int8)
        M, K = A.shape
        N = q.shape[1]
        Cm = np.empty((M, N), np.float32)
        self.lib.orc_matmul_int8(_p(A, np.float32), _p(q, np.int8), _p(s, np.float32), _p(Cm, np.float32),
                                 _sz(M), _sz(K), _sz(N), C.c_int(nthreads))
        return Cm

    def attn_decode(self, q, k_new, v_new, k_cache, v_cache, pos, scale, k_scale=None, v_scale=None,
                    nthreads=0):
        """GQA attention decode.  q [B][H][D], k_new/v_new [B][Hkv][D] fp32; caches
        [B][max_ctx][Hkv][D] as float32, uint16 (bf16 bits) or int8 (with scales
        [B][Hkv]), updated in place at pos.  Returns o [B][H][D]."""
        q, k_new, v_new = map(_f32, (q, k_new, v_new))
        B, H, D = q.shape
        Hkv = k_new.shape[1]
        max_ctx = k_cache.shape[1]
        dt = {np.dtype(np.float32): 0, np.dtype(np.uint16): 1, np.dtype(np.int8): 3}[k_cache.dtype]
        assert k_cache.flags["C_CONTIGUOUS"] and v_cache.flags["C_CONTIGUOUS"] and v_cache.dtype == k_cache.dtype
        ks = _f32(k_scale) if k_scale is not None else np.ones((B, Hkv), np.float32)
        vs = _f32(v_scale) if v_scale is not None else np.ones((B, Hkv), np.float32)
        o = np.empty((B, H, D), np.float32)
        self.lib.orc_attn_decode(_p(q, np.float32), _p(k_new, np.float32), _p(v_new, np.float32),
                                 k_cache.ctypes.data_as(C.c_void_p), v_cache.ctypes.data_as(C.c_void_p),
                                 _p(ks, np.float32), _p(vs, np.float32), _p(o, np.float32), _sz(B), _sz(H),
                                 _sz(Hkv), _sz(D), _sz(pos), _sz(max_ctx), C.c_float(scale), C.c_int(dt),
                                 C.c_int(nthreads))
        return o

    def e2e_decode(self, dims, is_gdn, weights, hidden_in, nthreads=0):
        """The end-to-end decode loop.  dims = (hidden, key_dim, value_dim, conv_dim, inter,
        full_heads, full_kv_heads, full_head_dim, layers); weights: dict of fp32 arrays named as
        the reference's Weights; hidden_in [T][B][hidden].  Returns (hidden_out, gdn_state
        [layers][B][value_dim])."""
        hin = _f32(hidden_in)
        T, B, H = hin.shape
        d = (C.c_size_t * 9)(*dims)
        g = np.ascontiguousarray(is_gdn, dtype=np.uint8)
        w = [_f32(weights[n]) for n in E2E_WEIGHTS]
        out = np.empty_like(hin)
        st = np.zeros((dims[8], B, dims[2]), np.float32)
        self.lib.orc_e2e_decode(d, g.ctypes.data_as(C.c_void_p), _sz(B), _sz(T), *[_p(x, np.float32) for x in w],
                                _p(hin, np.float32), _p(out, np.float32), _p(st, np.float32), C.c_int(nthreads))
        return out, st

    def chunk_wy(self, S, q, k, v, g, beta, scale=1.0, chunk=64, nthreads=0):
        """Chunked WY form in float64 (same layouts as delta_rule_seq)."""
        S = _f32(S).copy()
        q, k, v, g, beta = map(_f32, (q, k, v, g, beta))
        B, T, Hk, dk = q.shape
        Hv, dv = v.shape[2], v.shape[3]
        o = np.empty((B, T, Hv, dv), np.float32)
        self.lib.orc_chunk_wy_f64(_p(S, np.float32), _p(q, np.float32), _p(k, np.float32),
                                  _p(v, np.float32), _p(g, np.float32), _p(beta, np.float32),
                                  _p(o, np.float32), _sz(B), _sz(T), _sz(Hk), _sz(Hv), _sz(dk), _sz(dv),
                                  _sz(chunk), C.c_float(scale), C.c_int(nthreads))
        return S, o

    def num_threads(self) -> int:
        return int(self.lib.orc_num_threads())

    def set_threads(self, n: int) -> None:
        """OpenMP threads for later calls (of this library and of the reference's)."""
        self.lib.orc_set_threads(C.c_int(int(n)))


def _f16_to_u16(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, np.float32).astype(np.float16)).view(np.uint16)


def _u16_to_f32(a, kind: str) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint16)
    if kind == "f16":
        return a.view(np.float16).astype(np.float32)
    return (a.astype(np.uint32) << 16).view(np.float32)


E2E_WEIGHTS = ("g_q_proj", "g_k_proj", "g_v_proj", "g_o_proj", "g_conv_w", "g_beta", "f_q_proj", "f_k_proj",
               "f_v_proj", "f_o_proj", "gate_proj", "up_proj", "down_proj")


def e2e_weight_shapes(dims):
    """Shapes of the reference's Weights (row-major [in][out]; conv [4][conv_dim])."""
    H, KD, VD, CD, I, FH, FKV, FD = dims[:8]
    return {"g_q_proj": (H, KD), "g_k_proj": (H, KD), "g_v_proj": (H, VD), "g_o_proj": (VD, H),
            "g_conv_w": (4, CD), "g_beta": (KD,), "f_q_proj": (H, FH * FD), "f_k_proj": (H, FKV * FD),
            "f_v_proj": (H, FKV * FD), "f_o_proj": (FH * FD, H), "gate_proj": (H, I), "up_proj": (H, I),
            "down_proj": (I, H)}


def e2e_layer_pattern(layers):
    """Blocks of 3 GDN layers and 1 attention layer (gdn_e2e_decode.c:2414-2417)."""
    return np.array([1 if (l % 4) < 3 else 0 for l in range(layers)], np.uint8)


def f32_to_u16(a, kind: str) -> np.ndarray:
    """fp32 -> fp16 / bf16 bits, round to nearest even (bf16 rule of gdn_sve.c:81-88)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    if kind == "f16":
        return _f16_to_u16(a)
    u = a.view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


u16_to_f32 = _u16_to_f32

orc = _Oracle(_load(ORACLE_SO)) if ORACLE_SO.exists() else None
_ref_lib = _load(REF_SO)
ref = _Ref(_ref_lib) if _ref_lib is not None else None


class _RefInt8:
    """The reference's static int8 functions, exported by ref_int8_shim.c."""

    def __init__(self, lib):
        self.lib = lib

    def quantize_int8(self, B):
        B = _f32(B)
        K, N = B.shape
        q = np.empty((K, N), np.int8)
        s = np.empty((N,), np.float32)
        self.lib.ref_quantize_int8(_p(B, np.float32), _p(q, np.int8), _p(s, np.float32), _sz(K), _sz(N))
        return q, s

    def matmul_int8(self, A, q, s):
        A, s = _f32(A), _f32(s)
        q = np.ascontiguousarray(q, dtype=np.int8)
        M, K = A.shape
        N = q.shape[1]
        Cm = np.empty((M, N), np.float32)
        if M == 1:
            self.lib.ref_gemv_int8(_p(A, np.float32), _p(q, np.int8), _p(s, np.float32), _p(Cm, np.float32),
                                   _sz(K), _sz(N))
        else:
            self.lib.ref_gemm_int8(_p(A, np.float32), _p(q, np.int8), _p(s, np.float32), _p(Cm, np.float32),
                                   _sz(M), _sz(K), _sz(N))
        return Cm


class _RefAttn:
    """The reference's GQA attention decode (one sequence), via ref_attn_shim.c."""

    def __init__(self, lib, int8: bool):
        self.lib, self.int8 = lib, int8
        h, kvh, d = _sz(), _sz(), _sz()
        lib.ref_attn_geometry(C.byref(h), C.byref(kvh), C.byref(d))
        self.heads, self.kv_heads, self.head_dim = h.value, kvh.value, d.value

    def attn_decode(self, q, k_new, v_new, k_cache, v_cache, pos, k_scale=None, v_scale=None):
        """q [H*D], k_new/v_new [Hkv*D]; caches [max_ctx][Hkv*D] updated in place."""
        q, k_new, v_new = map(_f32, (q, k_new, v_new))
        o = np.empty(self.heads * self.head_dim, np.float32)
        ks = _f32(k_scale) if k_scale is not None else np.ones(self.kv_heads, np.float32)
        vs = _f32(v_scale) if v_scale is not None else np.ones(self.kv_heads, np.float32)
        self.lib.ref_attn_decode(_p(q, np.float32), _p(k_new, np.float32), _p(v_new, np.float32),
                                 k_cache.ctypes.data_as(C.c_void_p), v_cache.ctypes.data_as(C.c_void_p),
                                 _p(ks, np.float32), _p(vs, np.float32), _sz(pos), _sz(k_cache.shape[0]),
                                 _p(o, np.float32))
        return o


class _RefE2E:
    """The reference's end-to-end decode loop (0.8B geometry, int8 weights), via ref_e2e_shim.c."""

    def __init__(self, lib):
        self.lib = lib
        d = (C.c_size_t * 9)()
        lib.ref_e2e_geometry(d)
        self.dims = tuple(int(x) for x in d)

    def e2e_decode(self, weights, hidden_in):
        """hidden_in [T][hidden] -> (hidden_out [T][hidden], gdn_state [layers][value_dim])."""
        hin = _f32(hidden_in)
        out = np.empty_like(hin)
        st = np.zeros((self.dims[8], self.dims[2]), np.float32)
        w = [_f32(weights[n]) for n in E2E_WEIGHTS]
        self.lib.ref_e2e_decode(*[_p(x, np.float32) for x in w], _p(hin, np.float32), _p(out, np.float32),
                                _sz(hin.shape[0]), _p(st, np.float32))
        return out, st


_e2e_lib = _load(E2E_REF_SO)
ref_e2e = _RefE2E(_e2e_lib) if _e2e_lib is not None else None

_attn_lib = _load(ATTN_REF_SO)
ref_attn = _RefAttn(_attn_lib, False) if _attn_lib is not None else None
_attn_i8_lib = _load(ATTN_I8_REF_SO)
ref_attn_i8 = _RefAttn(_attn_i8_lib, True) if _attn_i8_lib is not None else None

_int8_lib = _load(INT8_REF_SO)
ref_int8 = _RefInt8(_int8_lib) if _int8_lib is not None else None


def require():
    """Return (orc, ref), building liboracle.so if it is missing."""
    global orc
    if orc is None:
        build(ref=False)
        orc = _Oracle(_load(ORACLE_SO))
    return orc, ref
