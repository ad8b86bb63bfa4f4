"""ctypes binding of libkai_gdn_cuda.so (the C ABI in include/kai_gdn_cuda.h).

The library is loaded from this package directory (built in-tree by
orionsbelt_b200/build.py).  There is no fallback: if the library is missing
or a symbol is absent, loading raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libkai_gdn_cuda.so"

OK, ERR_INVALID, ERR_CUDA, ERR_UNSUPPORTED, ERR_NOMEM, ERR_TIMEOUT = 0, 1, 2, 3, 4, 5
F32, BF16, F16, I8 = 0, 1, 2, 3

_sz = C.c_size_t
_vp = C.c_void_p
_i = C.c_int
_f = C.c_float


class DecodeArgs(C.Structure):
    """struct kai_gdn_decode_args."""
    _fields_ = [("state", _vp), ("q", _vp), ("k", _vp), ("v", _vp), ("g", _vp), ("beta", _vp), ("o", _vp),
                ("batch", _sz), ("heads_k", _sz), ("heads_v", _sz), ("dk", _sz), ("dv", _sz),
                ("scale", _f), ("in_dtype", _i), ("state_dtype", _i), ("out_dtype", _i)]


class Gdn2DecodeArgs(C.Structure):
    """struct kai_gdn2_decode_args."""
    _fields_ = [("state", _vp), ("q", _vp), ("k", _vp), ("v", _vp), ("g", _vp), ("b_gate", _vp), ("w_gate", _vp),
                ("o", _vp), ("batch", _sz), ("heads_k", _sz), ("heads_v", _sz), ("dk", _sz), ("dv", _sz),
                ("scale", _f), ("in_dtype", _i), ("state_dtype", _i), ("out_dtype", _i)]


class AttnDecodeArgs(C.Structure):
    """struct kai_gdn_attn_decode_args."""
    _fields_ = [("q", _vp), ("k_new", _vp), ("v_new", _vp), ("k_cache", _vp), ("v_cache", _vp), ("k_scale", _vp),
                ("v_scale", _vp), ("o", _vp), ("batch", _sz), ("heads", _sz), ("kv_heads", _sz), ("head_dim", _sz),
                ("pos", _sz), ("max_ctx", _sz), ("scale", _f), ("cache_dtype", _i)]


class AttnPrefillArgs(C.Structure):
    """struct kai_gdn_attn_prefill_args."""
    _fields_ = [("q", _vp), ("k_cache", _vp), ("v_cache", _vp), ("o", _vp), ("batch", _sz), ("T", _sz),
                ("heads", _sz), ("kv_heads", _sz), ("head_dim", _sz), ("pos0", _sz), ("max_ctx", _sz), ("scale", _f)]


class E2EConfig(C.Structure):
    """struct kai_gdn_e2e_config."""
    _fields_ = [("hidden", _sz), ("key_dim", _sz), ("value_dim", _sz), ("conv_dim", _sz), ("inter", _sz),
                ("full_heads", _sz), ("full_kv_heads", _sz), ("full_head_dim", _sz), ("layers", _sz),
                ("is_gdn", _vp), ("batch", _sz)]


class E2EWeights(C.Structure):
    """struct kai_gdn_e2e_weights."""
    _fields_ = [(n, _vp) for n in ("g_q_proj", "g_k_proj", "g_v_proj", "g_o_proj", "g_conv_w", "g_beta", "f_q_proj",
                                   "f_k_proj", "f_v_proj", "f_o_proj", "gate_proj", "up_proj", "down_proj")]


class ModelConfig(C.Structure):
    """struct kai_gdn_model_config."""
    _fields_ = [("hidden", _sz), ("layers", _sz), ("vocab", _sz), ("inter", _sz), ("is_gdn", _vp),
                ("gdn_heads_k", _sz), ("gdn_heads_v", _sz), ("gdn_head_dim", _sz), ("attn_heads", _sz),
                ("attn_kv_heads", _sz), ("attn_head_dim", _sz), ("rope_dims", _sz), ("rope_theta", _f),
                ("rms_eps", _f), ("batch", _sz), ("max_ctx", _sz), ("tp_rank", _i), ("tp_size", _i),
                ("nccl_id", _vp), ("seed", C.c_ulonglong), ("weight_std", _f)]


class ChunkArgs(C.Structure):
    """struct kai_gdn_chunk_args."""
    _fields_ = [("q", _vp), ("k", _vp), ("v", _vp), ("g", _vp), ("beta", _vp), ("state", _vp), ("o", _vp),
                ("batch", _sz), ("seq", _sz), ("heads_k", _sz), ("heads_v", _sz), ("dk", _sz), ("dv", _sz),
                ("chunk", _sz), ("scale", _f), ("in_dtype", _i), ("state_dtype", _i), ("out_dtype", _i)]


# name -> (restype, argtypes); every symbol declared in include/kai_gdn_cuda.h.
SIGNATURES = {
    # drop-in (void)
    "kai_run_gdn_cumdecay_f32_sve": (None, [_vp, _vp, _sz, _sz]),
    "kai_run_gdn_gated_scan_f32_sve": (None, [_vp, _vp, _vp, _vp, _sz, _sz]),
    "kai_run_gdn_causal_dwconv1d_f32_k4_sve": (None, [_vp, _vp, _vp, _vp, _sz, _sz]),
    "kai_run_gdn_gemv_f32_f32_f32_1x4_neon": (None, [_vp, _vp, _vp, _sz, _sz]),
    "gdn_cumdecay_f32": (None, [_vp, _vp, _sz, _sz]),
    "gdn_gated_scan_f32": (None, [_vp, _vp, _vp, _vp, _sz, _sz]),
    "gdn_causal_dwconv1d_f32": (None, [_vp, _vp, _vp, _vp, _sz, _sz]),
    "gdn_cumdecay_f16": (None, [_vp, _vp, _sz, _sz]),
    "gdn_gated_scan_f16": (None, [_vp, _vp, _vp, _vp, _sz, _sz]),
    "gdn_cumdecay_bf16": (None, [_vp, _vp, _sz, _sz]),
    "gdn_gated_scan_bf16": (None, [_vp, _vp, _vp, _vp, _sz, _sz]),
    "gdn2_gated_scan_f32": (None, [_vp, _vp, _vp, _vp, _vp, _vp, _sz, _sz]),
    "gdn_delta_rule_matmul": (None, [_vp, _vp, _vp, _sz, _sz, _sz]),
    # device, stream-ordered (int status)
    "kai_run_gdn_cumdecay_sm100a": (_i, [_vp, _vp, _i, _sz, _sz, _sz, _vp]),
    "kai_run_gdn_cumsum_f32_sm100a": (_i, [_vp, _vp, _sz, _sz, _sz, _vp]),
    "kai_run_gdn_gated_scan_sm100a": (_i, [_vp, _vp, _vp, _vp, _i, _sz, _sz, _sz, _vp]),
    "kai_run_gdn_gated_scan_noalloc_sm100a": (_i, [_vp, _vp, _vp, _vp, _i, _sz, _sz, _sz, _vp]),
    "kai_run_gdn2_gated_scan_f32_sm100a": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _sz, _sz, _sz, _vp]),
    "kai_run_gdn_causal_dwconv1d_k4_sm100a": (_i, [_vp, _vp, _vp, _vp, _i, _sz, _sz, _sz, _vp]),
    "kai_run_gdn_matmul_f32_sm100a": (_i, [_vp, _vp, _vp, _sz, _sz, _sz, _vp]),
    "kai_run_gdn_delta_rule_decode_sm100a": (_i, [C.POINTER(DecodeArgs), _vp]),
    "kai_run_gdn2_delta_rule_decode_sm100a": (_i, [C.POINTER(Gdn2DecodeArgs), _vp]),
    "kai_run_gdn_quantize_int8_sm100a": (_i, [_vp, _vp, _vp, _sz, _sz, _vp]),
    "kai_run_gdn_attention_decode_sm100a": (_i, [C.POINTER(AttnDecodeArgs), _vp]),
    "kai_run_gdn_attention_prefill_sm100a": (_i, [C.POINTER(AttnPrefillArgs), _vp]),
    "kai_gdn_e2e_create": (_i, [C.POINTER(E2EConfig), C.POINTER(E2EWeights), C.POINTER(_vp)]),
    "kai_gdn_e2e_step": (_i, [_vp, _vp, _vp, _vp]),
    "kai_gdn_e2e_state": (_i, [_vp, _sz, _vp, _vp]),
    "kai_gdn_e2e_destroy": (_i, [_vp]),
    "kai_run_gdn_matmul_int8_sm100a": (_i, [_vp, _vp, _vp, _vp, _sz, _sz, _sz, _vp]),
    "kai_gdn_int8_packed_bytes": (_sz, [_sz, _sz]),
    "kai_run_gdn_int8_pack_sm100a": (_i, [_vp, _vp, _sz, _sz, _vp]),
    "kai_run_gdn_matmul_int8_packed_sm100a": (_i, [_vp, _vp, _vp, _vp, _sz, _sz, _sz, _vp]),
    "kai_run_gdn_chunk_delta_rule_sm100a": (_i, [C.POINTER(ChunkArgs), _vp]),
    "kai_gdn_model_nccl_id": (_i, [_vp]),
    "kai_gdn_model_create": (_i, [C.POINTER(ModelConfig), C.POINTER(_vp)]),
    "kai_gdn_model_step": (_i, [_vp, _sz, _vp]),
    "kai_gdn_model_prefill": (_i, [_vp, _vp, _sz, _sz, _vp]),
    "kai_gdn_model_tokens": (_i, [_vp, _vp, _i]),
    "kai_gdn_model_read": (_i, [_vp, _i, _vp]),
    "kai_gdn_model_weight": (_i, [_vp, _sz, _i, _vp, _vp, C.POINTER(_sz), C.POINTER(_sz)]),
    "kai_gdn_model_fill": (_i, [_vp, _sz, C.c_ulonglong]),
    "kai_gdn_model_reset": (_i, [_vp]),
    "kai_gdn_model_destroy": (_i, [_vp]),
    # control
    "kai_gdn_cuda_set_device": (_i, [_i]),
    "kai_gdn_cuda_device_count": (_i, []),
    "kai_gdn_cuda_last_status": (_i, []),
    "kai_gdn_cuda_last_error": (C.c_char_p, []),
    "kai_gdn_cuda_clear_error": (None, []),
    "kai_gdn_cuda_version": (C.c_char_p, []),
    "kai_gdn_cuda_device_status": (C.c_int, [C.c_void_p]),
}


class GdnError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"kai_gdn_cuda status {status}: {msg}")
        self.status = status


_lib = None


def lib():
    """Load (once) and return the CDLL with every declared signature bound."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m orionsbelt_b200.build`")
        h = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name)  # AttributeError if the library lacks a declared symbol
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


def last_error() -> str:
    return (lib().kai_gdn_cuda_last_error() or b"").decode()


def check(status: int) -> None:
    """Raise GdnError for a non-zero status from a device entry point (and
    clear the thread's recorded failure, which the error now carries)."""
    if status != OK:
        msg = last_error()
        lib().kai_gdn_cuda_clear_error()
        raise GdnError(status, msg)


def check_dropin() -> None:
    """Raise if the drop-in (void) call just made on this thread recorded a
    failure (callers clear the record before the call: it keeps the last
    failure, not the last call's outcome)."""
    L = lib()
    st = L.kai_gdn_cuda_last_status()
    if st != OK:
        msg = last_error()
        L.kai_gdn_cuda_clear_error()
        raise GdnError(st, msg)
