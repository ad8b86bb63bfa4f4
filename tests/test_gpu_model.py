"""The config-4 decode engine (kai_gdn_model_*) against the CPU restatement
of its model (oracle/model.py), which composes the oracle's pinned int8
matmul, decode step and attention decode with the elementwise steps of the
reference's layer notes (docs/GDN_ARCHITECTURE_AUDIT.md sections 2-3).

A reduced geometry (two blocks of 3 GDN + 1 attention layer, hidden 256,
vocab 4096) runs six greedy steps of three and of six sequences,
teacher-forced with the oracle's own tokens so both sides see the same inputs
at every step.
Bars: hidden state and logits within 1e-3 relative L2 at every step (fp32
arithmetic in other orders through eight layers: int8 matmul sums, norms);
the engine's argmax equals the oracle's wherever the oracle's top two logits
differ by more than 1e-4 of the logit scale.

Tensor parallelism: the same model on two GPUs (tp_size 2, NCCL all-reduce
and all-gather), prompt prefill then decode steps, equals the single-GPU
engine (skipped with fewer than two GPUs).
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2
from orionsbelt_b200 import ops

pytestmark = pytest.mark.gpu

GEOM = dict(hidden=256, vocab=4096, inter=512, is_gdn=[1, 1, 1, 0, 1, 1, 1, 0], gdn_heads_k=2, gdn_heads_v=4,
            gdn_head_dim=128, attn_heads=4, attn_kv_heads=2, attn_head_dim=128, rope_dims=32, rope_theta=1e6,
            rms_eps=1e-6, max_ctx=64, weight_std=0.05)
B, STEPS = 3, 6
GEOM_TP = dict(GEOM, max_ctx=64 + STEPS)  # a 40-token prompt, then the steps


@pytest.mark.parametrize("B", [3, 6])
def test_model_matches_oracle(cuda, orc, B):
    """Batch 3 streams the layer projections with the CUDA-core GEMV, batch 6
    with the int8 tensor-core kernel; the LM head takes the tensor cores at
    every batch."""
    from oracle.model import ModelOracle, read_weights

    torch = cuda
    stream = torch.cuda.Stream()
    eng = ops.ModelEngine(GEOM, B, seed=11)
    W = read_weights(eng, GEOM)
    mo = ModelOracle(orc, GEOM, B, W)
    H, V = GEOM["hidden"], GEOM["vocab"]
    tok = np.array([5, 1000, 4095, 7, 2048, 1][:B], np.int32)
    with torch.cuda.stream(stream):
        for pos in range(STEPS):
            eng.set_tokens(tok)
            eng.step(pos, stream)  # eager, then graph capture, then replays
            stream.synchronize()
            got_tok = eng.tokens()
            got_h = eng.read(0, (B, H))
            got_l = eng.read(1, (B, V))
            h, logits, want_tok = mo.step(tok, pos)
            assert rel_l2(got_h, h) < 1e-3, (pos, rel_l2(got_h, h))
            assert rel_l2(got_l, logits) < 1e-3, (pos, rel_l2(got_l, logits))
            top2 = np.sort(logits, -1)[:, -2:]
            clear = (top2[:, 1] - top2[:, 0]) > 1e-4 * np.abs(logits).max()
            assert np.array_equal(got_tok[clear], want_tok[clear]), pos
            tok = want_tok  # teacher forcing with the oracle's tokens
    eng.close()


@pytest.mark.parametrize("B,split", [(2, None), (6, 40)])
def test_model_prefill_matches_oracle(cuda, orc, B, split):
    """A 70-token prompt (two 64-token chunks of the GDN scan, a partial last
    one) through kai_gdn_model_prefill -- in one call, or as 40 tokens and a
    continuation of 30 from position 40 -- equals the oracle stepping through
    the prompt token by token; then three decode steps from position 70."""
    from oracle.model import ModelOracle, read_weights

    torch = cuda
    geom = dict(GEOM, max_ctx=96)
    T, steps = 70, 3
    eng = ops.ModelEngine(geom, B, seed=13)
    W = read_weights(eng, geom)
    mo = ModelOracle(orc, geom, B, W)
    H, V = geom["hidden"], geom["vocab"]
    prompt = np.random.default_rng(B).integers(0, V, (B, T)).astype(np.int32)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        if split is None:
            eng.prefill(prompt, 0, stream)
        else:
            eng.prefill(prompt[:, :split], 0, stream)
            eng.prefill(prompt[:, split:], split, stream)
    for t in range(T):
        h, logits, want_tok = mo.step(prompt[:, t], t)
    got_h, got_l = eng.read(0, (B, H)), eng.read(1, (B, V))
    assert rel_l2(got_h, h) < 1e-3, rel_l2(got_h, h)
    assert rel_l2(got_l, logits) < 1e-3, rel_l2(got_l, logits)
    top2 = np.sort(logits, -1)[:, -2:]
    clear = (top2[:, 1] - top2[:, 0]) > 1e-4 * np.abs(logits).max()
    assert np.array_equal(eng.tokens()[clear], want_tok[clear])
    tok = want_tok
    with torch.cuda.stream(stream):
        for pos in range(T, T + steps):
            eng.set_tokens(tok)
            eng.step(pos, stream)
            stream.synchronize()
            h, logits, want_tok = mo.step(tok, pos)
            got_h, got_l = eng.read(0, (B, H)), eng.read(1, (B, V))
            assert rel_l2(got_h, h) < 1e-3, (pos, rel_l2(got_h, h))
            assert rel_l2(got_l, logits) < 1e-3, (pos, rel_l2(got_l, logits))
            tok = want_tok
    eng.close()


def _tp_rank(rank, nid, geom, prompt, tokens, q):
    try:
        import torch

        torch.cuda.set_device(rank)
        eng = ops.ModelEngine(geom, B, seed=11, tp_rank=rank, tp_size=2, nccl_id=nid)
        stream = torch.cuda.Stream()
        out = []
        with torch.cuda.stream(stream):
            eng.prefill(prompt, 0, stream)
            out.append((eng.tokens(), eng.read(0, (B, GEOM["hidden"])), eng.read(1, (B, GEOM["vocab"] // 2))))
            for pos, tok in enumerate(tokens, start=prompt.shape[1]):
                eng.set_tokens(tok)
                eng.step(pos, stream)
                stream.synchronize()
                out.append((eng.tokens(), eng.read(0, (B, GEOM["hidden"])),
                            eng.read(1, (B, GEOM["vocab"] // 2))))
        eng.close()
        q.put((rank, out))
    except Exception as exc:  # reported to the parent, which fails the test
        q.put((rank, f"error: {exc!r}"))


@pytest.mark.parametrize("kv_heads", [2, 1])
def test_model_tensor_parallel_two_gpus(cuda, kv_heads):
    """kv_heads 1 < tp_size: every rank keeps a copy of the one kv head (the
    path eight GPUs take with the config-4 model's four kv heads)."""
    torch = cuda
    geom = dict(GEOM_TP, attn_kv_heads=kv_heads)
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    rng = np.random.default_rng(4)
    prompt = rng.integers(0, GEOM["vocab"], (B, 40)).astype(np.int32)
    tokens = [rng.integers(0, GEOM["vocab"], B).astype(np.int32) for _ in range(STEPS)]
    nid = ops.ModelEngine.nccl_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_rank, args=(r, nid, geom, prompt, tokens, q)) for r in (0, 1)]
    for p in procs:
        p.start()
    try:
        res = dict(q.get(timeout=300) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in (0, 1):
        assert not isinstance(res[r], str), res[r]
    eng = ops.ModelEngine(geom, B, seed=11)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        eng.prefill(prompt, 0, stream)
        for i, tok in enumerate([None] + tokens):
            if tok is not None:
                eng.set_tokens(tok)
                eng.step(prompt.shape[1] + i - 1, stream)
                stream.synchronize()
            h = eng.read(0, (B, GEOM["hidden"]))
            lg = eng.read(1, (B, GEOM["vocab"]))
            t1 = eng.tokens()
            for r in (0, 1):
                tt, hh, ll = res[r][i]
                assert rel_l2(hh, h) < 1e-4, (i, r, rel_l2(hh, h))
                half = GEOM["vocab"] // 2
                assert rel_l2(ll, lg[:, r * half:(r + 1) * half]) < 1e-4
                assert np.array_equal(tt, t1)
    eng.close()
