"""Seeded synthetic inputs for the benchmark configurations (no dataset exists
for this path; every input is generated).

Distributions (one fixed seed per tensor, so any slice is reproducible):
  conv x ~ N(0,1) [T][Cc], conv w ~ N(0, 1/4) [4][Cc], hist = 0
  q, k ~ N(0,1), then L2-normalised per head (x / sqrt(|x|^2 + 1e-6))
  v ~ N(0,1)
  beta = sigmoid(N(0,1)),  g = -softplus(N(0,1)) * g_scale (0.1 in configs 0-2, 1 in 3)
  decode state ~ N(0, 0.02), prefill state = 0

`host_*` return float32 numpy arrays (small cases, parity tests, CPU samples);
`device_*` return CUDA tensors made by torch's seeded CUDA generator (full
benchmark sizes, generated in place in HBM).
"""
from __future__ import annotations

import numpy as np

CONFIGS = {
    0: dict(B=1, T=2048, Hk=16, Hv=32, dk=128, dv=128, g_scale=0.1, dtype="f32", state="f32"),
    1: dict(B=64, T=1, Hk=16, Hv=32, dk=128, dv=128, g_scale=0.1, dtype="bf16", state="f32", layers=24),
    2: dict(B=8, T=32768, Hk=16, Hv=32, dk=128, dv=128, g_scale=0.1, dtype="bf16", state="f32"),
    3: dict(B=32, T=8192, Hk=16, Hv=32, dk=128, dv=128, g_scale=1.0, dtype="bf16", state="f16"),
}


def conv_channels(Hk: int = 16, Hv: int = 32, d: int = 128) -> int:
    return (2 * Hk + Hv) * d


def _rng(seed: int, stream: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64([seed, stream]))


def softplus(x):
    return np.where(x > 20, x, np.log1p(np.exp(-np.abs(x))) + np.maximum(x, 0))


def l2norm(x, eps: float = 1e-6):
    x = np.asarray(x, np.float64)
    return (x / np.sqrt((x * x).sum(-1, keepdims=True) + eps)).astype(np.float32)


def host_gdn(B, T, Hk, Hv, dk, dv, g_scale=0.1, seed=0, state_std=0.0):
    """Inputs of the matrix-state delta rule, BTHD layouts, float32 numpy."""
    r = lambda i: _rng(seed, i)  # noqa: E731
    q = l2norm(r(1).standard_normal((B, T, Hk, dk)))
    k = l2norm(r(2).standard_normal((B, T, Hk, dk)))
    v = r(3).standard_normal((B, T, Hv, dv)).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-r(4).standard_normal((B, T, Hv))))).astype(np.float32)
    g = (-softplus(r(5).standard_normal((B, T, Hv))) * g_scale).astype(np.float32)
    S0 = (r(6).standard_normal((B, Hv, dk, dv)) * state_std).astype(np.float32)
    return dict(q=q, k=k, v=v, g=g, beta=beta, S0=S0)


def host_conv(T, C, seed=0, batch=None):
    r = lambda i: _rng(seed, 100 + i)  # noqa: E731
    shape = (T, C) if batch is None else (batch, T, C)
    x = r(1).standard_normal(shape).astype(np.float32)
    w = (r(2).standard_normal((4, C)) * 0.5).astype(np.float32)
    hshape = (3, C) if batch is None else (batch, 3, C)
    hist = np.zeros(hshape, np.float32)
    return x, w, hist


# ------------------------------------------------------------------ device

def _gen(seed: int, stream: int):
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed * 1000003 + stream)
    return g


def device_normal(shape, seed, stream, std=1.0, dtype=None):
    import torch
    t = torch.empty(shape, device="cuda", dtype=torch.float32)
    t.normal_(0.0, std, generator=_gen(seed, stream))
    return t if dtype is None else t.to(dtype)


def device_l2norm(x, eps=1e-6):
    import torch
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def device_gdn(B, T, Hk, Hv, dk, dv, g_scale=0.1, seed=0, in_dtype=None, state_std=0.0, state_dtype=None):
    """Full-size inputs generated in HBM (BTHD layouts)."""
    import torch
    in_dtype = in_dtype or torch.float32
    q = device_l2norm(device_normal((B, T, Hk, dk), seed, 1)).to(in_dtype)
    k = device_l2norm(device_normal((B, T, Hk, dk), seed, 2)).to(in_dtype)
    v = device_normal((B, T, Hv, dv), seed, 3, dtype=in_dtype)
    beta = torch.sigmoid(device_normal((B, T, Hv), seed, 4))
    g = -torch.nn.functional.softplus(device_normal((B, T, Hv), seed, 5)) * g_scale
    if state_std > 0:
        S0 = device_normal((B, Hv, dk, dv), seed, 6, std=state_std, dtype=state_dtype)
    else:
        S0 = torch.zeros((B, Hv, dk, dv), device="cuda", dtype=state_dtype or torch.float32)
    return dict(q=q, k=k, v=v, g=g.contiguous(), beta=beta.contiguous(), S0=S0)


def e2e_weight_shapes(dims):
    """Shapes of the end-to-end engine's weights, the reference's Weights
    (gdn_e2e_decode.c:1395-1424): row-major [in][out], conv weights
    [4][conv_dim], the GDN gate [key_dim].  dims = (hidden, key_dim,
    value_dim, conv_dim, inter, full_heads, full_kv_heads, full_head_dim, layers)."""
    H, KD, VD, CD, I, FH, FKV, FD = dims[:8]
    return {"g_q_proj": (H, KD), "g_k_proj": (H, KD), "g_v_proj": (H, VD), "g_o_proj": (VD, H),
            "g_conv_w": (4, CD), "g_beta": (KD,), "f_q_proj": (H, FH * FD), "f_k_proj": (H, FKV * FD),
            "f_v_proj": (H, FKV * FD), "f_o_proj": (FH * FD, H), "gate_proj": (H, I), "up_proj": (H, I),
            "down_proj": (I, H)}


def e2e_layer_pattern(layers):
    """Blocks of 3 GDN layers and 1 attention layer (gdn_e2e_decode.c:2414-2417)."""
    return np.array([1 if (l % 4) < 3 else 0 for l in range(layers)], np.uint8)

