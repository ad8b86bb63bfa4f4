"""CPU restatement of the config-4 decode engine (kai_gdn_model_*) -- TEST
INFRASTRUCTURE ONLY (a parity checker; the product never calls it).

The model is the Qwen3.5-style GDN hybrid of the reference's layer notes
(docs/GDN_ARCHITECTURE_AUDIT.md sections 2-3: in_proj_qkv / z / b / a,
Conv1D + SiLU, L2-normalised q and k, beta = sigmoid(b),
g = -exp(A_log) softplus(a + dt_bias), the delta-rule step, RMSNormGated,
out_proj; gated GQA attention with per-head q / k RMSNorm and partial RoPE)
in the block order of the reference's decode loop (gdn_e2e_decode.c:2775-2796:
layer, then SwiGLU FFN with residuals), with RMSNorm before each block,
embedding, final RMSNorm and a greedy LM head.  The heavy parts run on the
oracle's C restatements, each pinned to the reference elsewhere:
  int8 projections   orc_matmul_int8   (gemv_int8_neon / gemm_int8_neon)
  decode step        orc_delta_rule_decode (gpu/gdn_gpu_validate.c:100-118)
  attention decode   orc_attn_decode   (full_attn_real_forward, bf16 cache)
and the elementwise steps in float32 numpy.  The weights are the engine's
own int8 codes and scales, read back from a tensor-parallel size 1 engine.
Model-level parity is unpinned in the reference (it has no such model); the
checker pins the engine to these pinned pieces composed in this order.
"""
from __future__ import annotations

import numpy as np

from . import f32_to_u16

F = np.float32


def _silu(x):
    return (x / (F(1) + np.exp(-x))).astype(F)


def _rmsnorm(x, w, eps):
    ms = (x.astype(np.float64) ** 2).mean(-1, keepdims=True)
    return (x / np.sqrt(ms + eps).astype(F) * w).astype(F)


def _rope(x, pos, R, theta):
    """NeoX pairs (i, i + R/2) of the first R dims of x [..., D]."""
    if R == 0:
        return x
    half = R // 2
    j = np.arange(half, dtype=F)
    ang = (F(pos) * np.power(F(theta), -F(2) * j / F(R))).astype(F)
    c, s = np.cos(ang).astype(F), np.sin(ang).astype(F)
    y = x.copy()
    a, b = x[..., :half], x[..., half:R]
    y[..., :half] = a * c - b * s
    y[..., half:R] = a * s + b * c
    return y.astype(F)


class ModelOracle:
    """State and one greedy step of the model for `batch` sequences."""

    def __init__(self, orc, geom: dict, batch: int, weights: dict):
        self.orc, self.g, self.B = orc, dict(geom), int(batch)
        g = self.g
        self.is_gdn = [int(x) for x in g["is_gdn"]]
        self.w = weights  # {(layer, which): (codes or vector, scales)}
        d, hk, hv = g["gdn_head_dim"], g["gdn_heads_k"], g["gdn_heads_v"]
        self.C = (2 * hk + hv) * d
        B = self.B
        self.S, self.hist, self.kc, self.vc = {}, {}, {}, {}
        for l, isg in enumerate(self.is_gdn):
            if isg:
                self.S[l] = np.zeros((B, hv, d, d), F)
                self.hist[l] = np.zeros((B, 3, self.C), F)
            else:
                shape = (B, g["max_ctx"], g["attn_kv_heads"], g["attn_head_dim"])
                self.kc[l] = np.zeros(shape, np.uint16)
                self.vc[l] = np.zeros(shape, np.uint16)

    def _mm(self, x, key):
        q, s = self.w[key]
        return self.orc.matmul_int8(np.ascontiguousarray(x, F), q, s)

    def step(self, tokens, pos):
        """Returns (hidden [B][H], logits [B][V], next tokens [B])."""
        g, B = self.g, self.B
        eps = F(g["rms_eps"])
        eq, es = self.w[(0, "embed")]
        tok = np.asarray(tokens, np.int64)
        h = (eq[tok].astype(F) * es[tok][:, None]).astype(F)
        d, hk, hv = g["gdn_head_dim"], g["gdn_heads_k"], g["gdn_heads_v"]
        D, hq, hkv, R = g["attn_head_dim"], g["attn_heads"], g["attn_kv_heads"], g["rope_dims"]
        for l, isg in enumerate(self.is_gdn):
            x = _rmsnorm(h, self.w[(l, "norm_in")][0], eps)
            y = self._mm(x, (l, "in"))
            if isg:
                C = self.C
                cw = self.w[(l, "conv")][0].reshape(4, C)
                hs = self.hist[l]
                xc = y[:, :C]
                c = cw[0] * hs[:, 0]
                c = (c + cw[1] * hs[:, 1]).astype(F)
                c = (c + cw[2] * hs[:, 2]).astype(F)
                c = (c + cw[3] * xc).astype(F)
                hs[:, 0], hs[:, 1], hs[:, 2] = hs[:, 1].copy(), hs[:, 2].copy(), xc
                s = _silu(c)
                q = s[:, :hk * d].reshape(B, hk, d)
                k = s[:, hk * d:2 * hk * d].reshape(B, hk, d)
                v = np.ascontiguousarray(s[:, 2 * hk * d:].reshape(B, hv, d))
                q = (q / np.sqrt((q.astype(np.float64) ** 2).sum(-1, keepdims=True) + 1e-6)).astype(F)
                k = (k / np.sqrt((k.astype(np.float64) ** 2).sum(-1, keepdims=True) + 1e-6)).astype(F)
                zoff = C + hv * d
                bb, aa = y[:, zoff:zoff + hv], y[:, zoff + hv:zoff + 2 * hv]
                beta = (F(1) / (F(1) + np.exp(-bb))).astype(F)
                xa = (aa + self.w[(l, "dt_bias")][0]).astype(F)
                sp = np.where(xa > 20, xa, np.log1p(np.exp(np.minimum(xa, 20)))).astype(F)
                gg = (-np.exp(self.w[(l, "a_log")][0]) * sp).astype(F)
                self.S[l], o = self.orc.delta_rule_decode(self.S[l], np.ascontiguousarray(q),
                                                          np.ascontiguousarray(k), v, gg, beta,
                                                          scale=float(1.0 / np.sqrt(d)))
                z = y[:, C:C + hv * d].reshape(B, hv, d)
                o = (_rmsnorm(o, self.w[(l, "norm_gdn")][0], eps) * _silu(z)).astype(F)
                p = self._mm(o.reshape(B, hv * d), (l, "out"))
            else:
                qg = y[:, :hq * 2 * D].reshape(B, hq, 2 * D)
                qr, gate = qg[..., :D], qg[..., D:]
                kr = y[:, hq * 2 * D:hq * 2 * D + hkv * D].reshape(B, hkv, D)
                vr = np.ascontiguousarray(y[:, hq * 2 * D + hkv * D:].reshape(B, hkv, D))
                qn = _rope(_rmsnorm(qr, self.w[(l, "norm_q")][0], eps), pos, R, g["rope_theta"])
                kn = _rope(_rmsnorm(kr, self.w[(l, "norm_k")][0], eps), pos, R, g["rope_theta"])
                o = self.orc.attn_decode(np.ascontiguousarray(qn), np.ascontiguousarray(kn), vr, self.kc[l],
                                         self.vc[l], pos, float(1.0 / np.sqrt(D)))
                o = (o * (F(1) / (F(1) + np.exp(-gate)))).astype(F)
                p = self._mm(o.reshape(B, hq * D), (l, "out"))
            h = (h + p).astype(F)
            x = _rmsnorm(h, self.w[(l, "norm_post")][0], eps)
            gu = self._mm(x, (l, "gate_up"))
            I = gu.shape[1] // 2
            act = (_silu(gu[:, :I]) * gu[:, I:]).astype(F)
            h = (h + self._mm(act, (l, "down"))).astype(F)
        x = _rmsnorm(h, self.w[(0, "norm_final")][0], eps)
        logits = self._mm(x, (0, "lm"))
        return h, logits, logits.argmax(-1).astype(np.int32)


def read_weights(engine, geom) -> dict:
    """All weights of a tensor-parallel size 1 engine, keyed for ModelOracle."""
    E = type(engine)
    out = {}
    for l, isg in enumerate(geom["is_gdn"]):
        for name, which in (("in", E.W_IN), ("out", E.W_OUT), ("gate_up", E.W_GATE_UP), ("down", E.W_DOWN),
                            ("norm_in", E.V_NORM_IN), ("norm_post", E.V_NORM_POST)):
            out[(l, name)] = engine.weight(l, which)
        if isg:
            for name, which in (("conv", E.V_CONV), ("a_log", E.V_A_LOG), ("dt_bias", E.V_DT_BIAS),
                                ("norm_gdn", E.V_NORM_GDN)):
                out[(l, name)] = engine.weight(l, which)
        else:
            for name, which in (("norm_q", E.V_NORM_Q), ("norm_k", E.V_NORM_K)):
                out[(l, name)] = engine.weight(l, which)
    out[(0, "lm")] = engine.weight(0, E.W_LM)
    out[(0, "norm_final")] = engine.weight(0, E.V_NORM_FINAL)
    out[(0, "embed")] = engine.weight(0, E.W_EMBED)
    return out


__all__ = ["ModelOracle", "read_weights", "f32_to_u16"]
