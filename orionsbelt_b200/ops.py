"""Python mirror of the kai GDN operator interface over libkai_gdn_cuda.so.

Two layers, both calling the C ABI (include/kai_gdn_cuda.h) through ctypes:

* The drop-in names take numpy arrays (host memory) exactly like the reference
  C functions take host pointers: ``kai_run_gdn_cumdecay_f32_sve(a, decay)``
  fills ``decay`` in place, ``state`` / ``hist`` are updated in place, and the
  call returns when the result is there (kleidiai_submission/kai/ukernels/gdn/
  *.h, src/orionsbelt/engines/cpu/kernels/gdn_sve.h, gdn_delta_matmul.h).
* The device layer takes CUDA tensors (torch is used only to own device memory
  and streams) and launches on the current torch stream: ``cumdecay``,
  ``cumsum``, ``gated_scan``, ``gdn2_gated_scan``, ``causal_dwconv1d``,
  ``matmul``, ``quantize_int8``, ``matmul_int8``, ``pack_int8``, ``matmul_int8_packed``, ``attention_prefill``, ``attention_decode``, ``E2EEngine``, ``delta_rule_decode``,
  ``gdn2_delta_rule_decode`` and ``chunk_delta_rule``.

There is no CPU fallback anywhere: a missing library raises at import of the
first call, and every failed call raises GdnError with the library's message.
"""
from __future__ import annotations

import numpy as np

from . import _lib
from ._lib import BF16, F16, F32, check, check_dropin, lib

# ----------------------------------------------------------------- drop-in


def _host(a: np.ndarray, dtype=np.float32) -> int:
    if not isinstance(a, np.ndarray) or a.dtype != dtype or not a.flags["C_CONTIGUOUS"]:
        raise TypeError(f"expected a C-contiguous numpy {np.dtype(dtype).name} array")
    return a.ctypes.data


def kai_run_gdn_cumdecay_f32_sve(a: np.ndarray, decay: np.ndarray) -> None:
    seq, ch = a.shape
    lib().kai_gdn_cuda_clear_error()  # a failure recorded earlier is not this call's
    lib().kai_run_gdn_cumdecay_f32_sve(_host(a), _host(decay), seq, ch)
    check_dropin()


def kai_run_gdn_gated_scan_f32_sve(g, x, s, state) -> None:
    seq, ch = x.shape
    lib().kai_gdn_cuda_clear_error()  # a failure recorded earlier is not this call's
    lib().kai_run_gdn_gated_scan_f32_sve(_host(g), _host(x), _host(s), _host(state), seq, ch)
    check_dropin()


def kai_run_gdn_causal_dwconv1d_f32_k4_sve(x, w, out, hist) -> None:
    seq, ch = x.shape
    lib().kai_gdn_cuda_clear_error()  # a failure recorded earlier is not this call's
    lib().kai_run_gdn_causal_dwconv1d_f32_k4_sve(_host(x), _host(w), _host(out), _host(hist), seq, ch)
    check_dropin()


def kai_run_gdn_gemv_f32_f32_f32_1x4_neon(a, b, c) -> None:
    k, n = b.shape
    lib().kai_gdn_cuda_clear_error()  # a failure recorded earlier is not this call's
    lib().kai_run_gdn_gemv_f32_f32_f32_1x4_neon(_host(a), _host(b), _host(c), k, n)
    check_dropin()


def gdn_delta_rule_matmul(A, B, Cm) -> None:
    M, K = A.shape
    N = B.shape[1]
    lib().kai_gdn_cuda_clear_error()  # a failure recorded earlier is not this call's
    lib().gdn_delta_rule_matmul(_host(A), _host(B), _host(Cm), M, K, N)
    check_dropin()


def gdn_cumdecay_narrow(a, decay_u16, kind: str) -> None:
    seq, ch = a.shape
    lib().kai_gdn_cuda_clear_error()  # a failure recorded earlier is not this call's
    getattr(lib(), "gdn_cumdecay_" + kind)(_host(a), _host(decay_u16, np.uint16), seq, ch)
    check_dropin()


def gdn_gated_scan_narrow(g, x, s, state_u16, kind: str) -> None:
    seq, ch = x.shape
    lib().kai_gdn_cuda_clear_error()  # a failure recorded earlier is not this call's
    getattr(lib(), "gdn_gated_scan_" + kind)(_host(g), _host(x), _host(s), _host(state_u16, np.uint16), seq, ch)
    check_dropin()


def gdn2_gated_scan_f32(g, b_gate, w_gate, x, s, state) -> None:
    seq, ch = x.shape
    lib().kai_gdn_cuda_clear_error()  # a failure recorded earlier is not this call's
    lib().gdn2_gated_scan_f32(_host(g), _host(b_gate), _host(w_gate), _host(x), _host(s), _host(state), seq, ch)
    check_dropin()


# ------------------------------------------------------------ device layer

def _torch():
    import torch
    return torch


def _dt(t) -> int:
    torch = _torch()
    return {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}[t.dtype]


def _dev(t, *, dtype=None) -> int:
    torch = _torch()
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"expected {dtype}, got {t.dtype}")
    return t.data_ptr()


def _stream(stream=None) -> int:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def cumdecay(a, decay, stream=None) -> None:
    """a [batch][seq][ch] fp32 -> decay (fp32 / fp16 / bf16) prefix product."""
    torch = _torch()
    b, s, c = a.shape if a.dim() == 3 else (1, *a.shape)
    check(lib().kai_run_gdn_cumdecay_sm100a(_dev(a, dtype=torch.float32), _dev(decay), _dt(decay), b, s, c,
                                            _stream(stream)))


def cumsum(g, gcum, stream=None) -> None:
    torch = _torch()
    b, s, c = g.shape if g.dim() == 3 else (1, *g.shape)
    check(lib().kai_run_gdn_cumsum_f32_sm100a(_dev(g, dtype=torch.float32), _dev(gcum, dtype=torch.float32),
                                              b, s, c, _stream(stream)))


def gated_scan(g, x, s, state, stream=None) -> None:
    torch = _torch()
    b, t, c = x.shape if x.dim() == 3 else (1, *x.shape)
    f = torch.float32
    check(lib().kai_run_gdn_gated_scan_sm100a(_dev(g, dtype=f), _dev(x, dtype=f), _dev(s, dtype=f), _dev(state),
                                              _dt(state), b, t, c, _stream(stream)))


def gdn2_gated_scan(g, b_gate, w_gate, x, s, state, stream=None) -> None:
    torch = _torch()
    b, t, c = x.shape if x.dim() == 3 else (1, *x.shape)
    f = torch.float32
    check(lib().kai_run_gdn2_gated_scan_f32_sm100a(_dev(g, dtype=f), _dev(b_gate, dtype=f), _dev(w_gate, dtype=f),
                                                   _dev(x, dtype=f), _dev(s, dtype=f), _dev(state, dtype=f),
                                                   b, t, c, _stream(stream)))


def causal_dwconv1d(x, w, out, hist, stream=None) -> None:
    """x, out [batch][seq][ch], hist [batch][3][ch] (same dtype), w [4][ch] fp32."""
    torch = _torch()
    b, t, c = x.shape if x.dim() == 3 else (1, *x.shape)
    if out.dtype != x.dtype or hist.dtype != x.dtype:
        raise TypeError("x, out and hist must share a dtype")
    check(lib().kai_run_gdn_causal_dwconv1d_k4_sm100a(_dev(x), _dev(w, dtype=torch.float32), _dev(out), _dev(hist),
                                                      _dt(x), b, t, c, _stream(stream)))


def matmul(A, B, Cm, stream=None) -> None:
    torch = _torch()
    f = torch.float32
    M, K = A.shape
    N = B.shape[1]
    check(lib().kai_run_gdn_matmul_f32_sm100a(_dev(A, dtype=f), _dev(B, dtype=f), _dev(Cm, dtype=f), M, K, N,
                                              _stream(stream)))


def quantize_int8(B, q, s, stream=None) -> None:
    """B [K][N] fp32 -> q [K][N] int8, s [N] fp32 (per-column symmetric scale),
    bit-identical to quantize_weight (gdn_e2e_decode.c:175-199)."""
    torch = _torch()
    K, N = B.shape
    check(lib().kai_run_gdn_quantize_int8_sm100a(_dev(B, dtype=torch.float32), _dev(q, dtype=torch.int8),
                                                 _dev(s, dtype=torch.float32), K, N, _stream(stream)))


def matmul_int8(A, q, s, Cm, stream=None) -> None:
    """Cm [M][N] = (A [M][K] . q [K][N]) * s[n]: matmul_int8 (gdn_e2e_decode.c:681)."""
    torch = _torch()
    f = torch.float32
    M, K = A.shape
    N = q.shape[1]
    check(lib().kai_run_gdn_matmul_int8_sm100a(_dev(A, dtype=f), _dev(q, dtype=torch.int8), _dev(s, dtype=f),
                                               _dev(Cm, dtype=f), M, K, N, _stream(stream)))


def pack_int8(q, stream=None):
    """The streaming layout of q [K][N] int8 for matmul_int8_packed (a new
    uint8 device tensor; the reference prepares its QW weights once at load
    the same way, quantize_weight, gdn_e2e_decode.c:175-199)."""
    torch = _torch()
    K, N = q.shape
    nbytes = lib().kai_gdn_int8_packed_bytes(K, N)
    if nbytes == 0:
        raise ValueError(f"pack_int8: N % 16 must be zero and K <= 131072 (K={K}, N={N})")
    qp = torch.empty(nbytes, dtype=torch.uint8, device=q.device)
    check(lib().kai_run_gdn_int8_pack_sm100a(_dev(q, dtype=torch.int8), qp.data_ptr(), K, N, _stream(stream)))
    return qp


def matmul_int8_packed(A, qp, s, Cm, stream=None) -> None:
    """Cm [M][N] = (A [M][K] . q) * s[n] over qp = pack_int8(q), on the tensor
    cores (16 rows of A per pass over the weights)."""
    torch = _torch()
    f = torch.float32
    M, K = A.shape
    N = Cm.shape[1]
    check(lib().kai_run_gdn_matmul_int8_packed_sm100a(_dev(A, dtype=f), qp.data_ptr(), _dev(s, dtype=f),
                                                      _dev(Cm, dtype=f), M, K, N, _stream(stream)))


def attn_decode_args(q, k_new, v_new, k_cache, v_cache, o, pos: int, scale: float, k_scale=None,
                     v_scale=None) -> _lib.AttnDecodeArgs:
    """Pack struct kai_gdn_attn_decode_args: q [B][H][D], k_new/v_new [B][Hkv][D] fp32,
    caches [B][max_ctx][Hkv][D] (fp32, bf16 or int8 with scales [B][Hkv]), o [B][H][D]."""
    torch = _torch()
    f = torch.float32
    B, H, D = q.shape
    Hkv, max_ctx = k_new.shape[1], k_cache.shape[1]
    if k_cache.dtype != v_cache.dtype:
        raise TypeError("k_cache and v_cache must share a dtype")
    dt = {torch.float32: F32, torch.bfloat16: BF16, torch.int8: _lib.I8}[k_cache.dtype]
    ks = _dev(k_scale, dtype=f) if dt == _lib.I8 else None
    vs = _dev(v_scale, dtype=f) if dt == _lib.I8 else None
    return _lib.AttnDecodeArgs(_dev(q, dtype=f), _dev(k_new, dtype=f), _dev(v_new, dtype=f), _dev(k_cache),
                               _dev(v_cache), ks, vs, _dev(o, dtype=f), B, H, Hkv, D, int(pos), max_ctx,
                               float(scale), dt)


def attention_decode(q, k_new, v_new, k_cache, v_cache, o, pos: int, scale: float, k_scale=None, v_scale=None,
                     stream=None) -> None:
    """GQA attention decode with KV-cache append (gdn_e2e_decode.c:1532-1634, int8 cache :1652-1830)."""
    args = attn_decode_args(q, k_new, v_new, k_cache, v_cache, o, pos, scale, k_scale, v_scale)
    check(lib().kai_run_gdn_attention_decode_sm100a(args, _stream(stream)))


def attention_prefill(q, k_cache, v_cache, o, pos0: int, scale: float, stream=None) -> None:
    """Causal GQA attention of a prompt over bf16 caches that already hold its
    keys and values: q, o [B][T][H][D] fp32, caches [B][max_ctx][Hkv][D]; query
    t attends to positions 0 .. pos0 + t."""
    torch = _torch()
    f = torch.float32
    B, T, H, D = q.shape
    Hkv, max_ctx = k_cache.shape[2], k_cache.shape[1]
    args = _lib.AttnPrefillArgs(_dev(q, dtype=f), _dev(k_cache, dtype=torch.bfloat16),
                                _dev(v_cache, dtype=torch.bfloat16), _dev(o, dtype=f), B, T, H, Hkv, D, int(pos0),
                                max_ctx, float(scale))
    check(lib().kai_run_gdn_attention_prefill_sm100a(args, _stream(stream)))


class E2EEngine:
    """The end-to-end hybrid decode engine (kai_gdn_e2e_*): the reference's decode loop
    (gdn_e2e_decode.c:2775-2796) for `batch` sequences.  dims = (hidden, key_dim, value_dim,
    conv_dim, inter, full_heads, full_kv_heads, full_head_dim, layers); weights: dict of host
    fp32 numpy arrays named as the reference's Weights."""

    NAMES = ("g_q_proj", "g_k_proj", "g_v_proj", "g_o_proj", "g_conv_w", "g_beta", "f_q_proj", "f_k_proj",
             "f_v_proj", "f_o_proj", "gate_proj", "up_proj", "down_proj")

    def __init__(self, dims, is_gdn, batch: int, weights):
        import ctypes as C
        self._is_gdn = np.ascontiguousarray(is_gdn, dtype=np.uint8)
        self.dims, self.batch = tuple(int(x) for x in dims), int(batch)
        H, KD, VD, CD, I, FH, FKV, FD, L = self.dims
        cfg = _lib.E2EConfig(H, KD, VD, CD, I, FH, FKV, FD, L, self._is_gdn.ctypes.data, self.batch)
        arrs = [np.ascontiguousarray(weights[n], dtype=np.float32) for n in self.NAMES]
        w = _lib.E2EWeights(*[a.ctypes.data for a in arrs])
        h = C.c_void_p()
        check(lib().kai_gdn_e2e_create(cfg, w, C.byref(h)))
        self._h = h

    def step(self, hidden_in, hidden_out, stream=None) -> None:
        """hidden_in, hidden_out: [batch][hidden] fp32 CUDA tensors."""
        torch = _torch()
        check(lib().kai_gdn_e2e_step(self._h, _dev(hidden_in, dtype=torch.float32),
                                     _dev(hidden_out, dtype=torch.float32), _stream(stream)))

    def gdn_state(self, layer: int):
        st = np.empty((self.batch, self.dims[2]), np.float32)
        check(lib().kai_gdn_e2e_state(self._h, layer, st.ctypes.data, None))
        return st

    def close(self) -> None:
        if self._h:
            lib().kai_gdn_e2e_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ModelEngine:
    """Decode engine of a Qwen3.5-style GDN hybrid (kai_gdn_model_*), optionally
    tensor-parallel: `geom` is a dict of the kai_gdn_model_config fields
    (hidden, layers, vocab, inter, is_gdn, gdn_heads_k, gdn_heads_v, gdn_head_dim,
    attn_heads, attn_kv_heads, attn_head_dim, rope_dims, rope_theta, rms_eps,
    max_ctx, weight_std); tp_rank / tp_size / nccl_id place it in a
    tensor-parallel group (nccl_id: bytes from nccl_id(), made by one rank and
    shared with the others; an id serves one engine's communicator)."""

    W_IN, W_OUT, W_GATE_UP, W_DOWN = 0, 1, 2, 3
    V_NORM_IN, V_NORM_POST, V_CONV, V_A_LOG, V_DT_BIAS, V_NORM_GDN, V_NORM_Q, V_NORM_K = 4, 5, 6, 7, 8, 9, 10, 11
    W_LM, V_NORM_FINAL, W_EMBED = 12, 13, 14

    @staticmethod
    def nccl_id() -> bytes:
        import ctypes as C
        buf = C.create_string_buffer(128)
        check(lib().kai_gdn_model_nccl_id(buf))
        return buf.raw

    def __init__(self, geom: dict, batch: int, seed: int = 1, tp_rank: int = 0, tp_size: int = 1,
                 nccl_id: bytes | None = None):
        import ctypes as C
        g = dict(geom)
        self._is_gdn = np.ascontiguousarray(g.pop("is_gdn"), dtype=np.uint8)
        self._nid = C.create_string_buffer(nccl_id, 128) if nccl_id is not None else None
        self.batch = int(batch)
        self.geom = dict(geom)
        cfg = _lib.ModelConfig(g["hidden"], len(self._is_gdn), g["vocab"], g["inter"], self._is_gdn.ctypes.data,
                               g["gdn_heads_k"], g["gdn_heads_v"], g["gdn_head_dim"], g["attn_heads"],
                               g["attn_kv_heads"], g["attn_head_dim"], g["rope_dims"], float(g["rope_theta"]),
                               float(g["rms_eps"]), self.batch, g["max_ctx"], int(tp_rank), int(tp_size),
                               C.cast(self._nid, C.c_void_p) if self._nid is not None else None, int(seed),
                               float(g.get("weight_std", 0.0)))
        h = C.c_void_p()
        check(lib().kai_gdn_model_create(C.byref(cfg), C.byref(h)))
        self._h = h

    def set_tokens(self, tokens) -> None:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        check(lib().kai_gdn_model_tokens(self._h, t.ctypes.data, 1))

    def tokens(self) -> np.ndarray:
        t = np.empty(self.batch, np.int32)
        check(lib().kai_gdn_model_tokens(self._h, t.ctypes.data, 0))
        return t

    def step(self, pos: int, stream=None) -> None:
        check(lib().kai_gdn_model_step(self._h, int(pos), _stream(stream)))

    def reset(self) -> None:
        """Every sequence back to position 0 (GDN states and conv histories zero)."""
        check(lib().kai_gdn_model_reset(self._h))

    def prefill(self, tokens, pos0: int = 0, stream=None) -> None:
        """Consume prompts tokens [batch][T] at positions pos0 .. pos0 + T - 1;
        the greedy next tokens become the current tokens."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        if t.ndim != 2 or t.shape[0] != self.batch:
            raise ValueError(f"prefill: tokens must be [batch={self.batch}][T], got {t.shape}")
        check(lib().kai_gdn_model_prefill(self._h, t.ctypes.data, t.shape[1], int(pos0), _stream(stream)))

    def read(self, what: int, shape) -> np.ndarray:
        out = np.empty(shape, np.float32)
        check(lib().kai_gdn_model_read(self._h, what, out.ctypes.data))
        return out

    def weight(self, layer: int, which: int):
        """(codes or vector, scales or None) of this rank's weight `which` of `layer`."""
        import ctypes as C
        rows, cols = C.c_size_t(), C.c_size_t()
        check(lib().kai_gdn_model_weight(self._h, layer, which, None, None, C.byref(rows), C.byref(cols)))
        r, c = rows.value, cols.value
        if which in (self.W_IN, self.W_OUT, self.W_GATE_UP, self.W_DOWN, self.W_LM, self.W_EMBED):
            q = np.empty((r, c), np.int8)
            s = np.empty(r if which == self.W_EMBED else c, np.float32)
            check(lib().kai_gdn_model_weight(self._h, layer, which, q.ctypes.data, s.ctypes.data, C.byref(rows),
                                             C.byref(cols)))
            return q, s
        v = np.empty(c, np.float32)
        check(lib().kai_gdn_model_weight(self._h, layer, which, v.ctypes.data, None, C.byref(rows), C.byref(cols)))
        return v, None

    def fill(self, ctx: int, seed: int = 7) -> None:
        check(lib().kai_gdn_model_fill(self._h, int(ctx), int(seed)))

    def close(self) -> None:
        if self._h:
            lib().kai_gdn_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def decode_args(state, q, k, v, g, beta, o, scale: float) -> _lib.DecodeArgs:
    """Pack struct kai_gdn_decode_args from tensors:
    state [B][Hv][dk][dv], q,k [B][Hk][dk], v [B][Hv][dv], g,beta [B][Hv], o [B][Hv][dv]."""
    torch = _torch()
    B, Hv, dk, dv = state.shape
    Hk = q.shape[1]
    if q.dtype != k.dtype or v.dtype != q.dtype:
        raise TypeError("q, k, v must share a dtype")
    return _lib.DecodeArgs(_dev(state), _dev(q), _dev(k), _dev(v), _dev(g, dtype=torch.float32),
                           _dev(beta, dtype=torch.float32), _dev(o), B, Hk, Hv, dk, dv, float(scale),
                           _dt(q), _dt(state), _dt(o))


def delta_rule_decode(state, q, k, v, g, beta, o, scale: float = 1.0, stream=None) -> None:
    """One token of the matrix-state gated delta rule for every (batch, value head)."""
    args = decode_args(state, q, k, v, g, beta, o, scale)
    check(lib().kai_run_gdn_delta_rule_decode_sm100a(args, _stream(stream)))


def gdn2_decode_args(state, q, k, v, g, b_gate, w_gate, o, scale: float) -> _lib.Gdn2DecodeArgs:
    """Pack struct kai_gdn2_decode_args from tensors: state [B][Hv][dk][dv],
    q,k [B][Hk][dk], v [B][Hv][dv], g,b_gate [B][Hv][dk], w_gate [B][Hv][dv], o [B][Hv][dv]."""
    torch = _torch()
    B, Hv, dk, dv = state.shape
    Hk = q.shape[1]
    if q.dtype != k.dtype or v.dtype != q.dtype:
        raise TypeError("q, k, v must share a dtype")
    f = torch.float32
    return _lib.Gdn2DecodeArgs(_dev(state), _dev(q), _dev(k), _dev(v), _dev(g, dtype=f), _dev(b_gate, dtype=f),
                               _dev(w_gate, dtype=f), _dev(o), B, Hk, Hv, dk, dv, float(scale), _dt(q), _dt(state),
                               _dt(o))


def gdn2_delta_rule_decode(state, q, k, v, g, b_gate, w_gate, o, scale: float = 1.0, stream=None) -> None:
    """One token of the GDN-2 recurrence (per-channel decay, erase and write gates)
    for every (batch, value head); bench/gdn2_reference.py:58-145."""
    args = gdn2_decode_args(state, q, k, v, g, b_gate, w_gate, o, scale)
    check(lib().kai_run_gdn2_delta_rule_decode_sm100a(args, _stream(stream)))


def chunk_args(q, k, v, g, beta, state, o, scale: float, chunk: int = 64) -> _lib.ChunkArgs:
    """Pack struct kai_gdn_chunk_args: q,k [B][T][Hk][dk], v [B][T][Hv][dv],
    g,beta [B][T][Hv], state [B][Hv][dk][dv], o [B][T][Hv][dv]."""
    torch = _torch()
    B, T, Hk, dk = q.shape
    Hv, dv = v.shape[2], v.shape[3]
    if q.dtype != k.dtype or v.dtype != q.dtype:
        raise TypeError("q, k, v must share a dtype")
    return _lib.ChunkArgs(_dev(q), _dev(k), _dev(v), _dev(g, dtype=torch.float32), _dev(beta, dtype=torch.float32),
                          _dev(state), _dev(o), B, T, Hk, Hv, dk, dv, chunk, float(scale),
                          _dt(q), _dt(state), _dt(o))


def chunk_delta_rule(q, k, v, g, beta, state, o, scale: float = 1.0, chunk: int = 64, stream=None) -> None:
    """Chunkwise WY gated delta-rule scan over the whole sequence (state in/out)."""
    args = chunk_args(q, k, v, g, beta, state, o, scale, chunk)
    check(lib().kai_run_gdn_chunk_delta_rule_sm100a(args, _stream(stream)))
