"""The multi-GPU partition, on CPU: world-size-2 gloo ranks each run their
shard of the decode step and of the chunked scan through the oracle; the
all-gathered results equal the unsharded run, and the timing reduction is the
max over ranks (the only collective the benchmark uses)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from orionsbelt_b200 import shard


def test_batch_and_head_slices_partition():
    for n in (1, 2, 3, 4, 8):
        cover = []
        for r in range(n):
            a, b = shard.batch_slice(64, n, r)
            cover.extend(range(a, b))
        assert cover == list(range(64))
        vs, ks = [], []
        for r in range(n if n <= 16 else 16):
            (v0, v1), (k0, k1) = shard.head_slice(32, 16, n, r)
            assert (v0, v1) == (2 * k0, 2 * k1)  # a rank owns both value heads of each key head
            vs.extend(range(v0, v1))
            ks.extend(range(k0, k1))
        assert vs == list(range(32)) and ks == list(range(16))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    import oracle
    from orionsbelt_b200 import synth

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    orc, _ = oracle.require()
    # decode step, batch-sharded
    B, Hk, Hv, d = 6, 2, 4, 32
    full = synth.host_gdn(B, 1, Hk, Hv, d, d, seed=3, state_std=0.05)
    b0, b1 = shard.batch_slice(B, world, rank)
    S, o = orc.delta_rule_decode(full["S0"][b0:b1], full["q"][b0:b1, 0], full["k"][b0:b1, 0], full["v"][b0:b1, 0],
                                 full["g"][b0:b1, 0], full["beta"][b0:b1, 0], scale=0.5, nthreads=1)
    parts = [None] * world
    dist.all_gather_object(parts, (S, o))
    # chunked scan, head-sharded
    dd = synth.host_gdn(1, 70, Hk, Hv, d, d, seed=4, state_std=0.05)
    (v0, v1), (k0, k1) = shard.head_slice(Hv, Hk, world, rank)
    S2, o2 = orc.chunk_wy(dd["S0"][:, v0:v1], dd["q"][:, :, k0:k1], dd["k"][:, :, k0:k1], dd["v"][:, :, v0:v1],
                          dd["g"][:, :, v0:v1], dd["beta"][:, :, v0:v1], scale=0.5, nthreads=1)
    heads = [None] * world
    dist.all_gather_object(heads, (S2, o2))
    # timing reduction: max over ranks
    t = torch.tensor([1.0 + rank])
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    if rank == 0:
        q.put((parts, heads, float(t.item())))
    dist.barrier()
    dist.destroy_process_group()


def test_world_size_2_shards_equal_unsharded_run():
    import oracle
    from orionsbelt_b200 import synth

    orc, _ = oracle.require()
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    parts, heads, tmax = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    B, Hk, Hv, d = 6, 2, 4, 32
    full = synth.host_gdn(B, 1, Hk, Hv, d, d, seed=3, state_std=0.05)
    S, o = orc.delta_rule_decode(full["S0"], full["q"][:, 0], full["k"][:, 0], full["v"][:, 0], full["g"][:, 0],
                                 full["beta"][:, 0], scale=0.5, nthreads=1)
    assert np.array_equal(np.concatenate([p[0] for p in parts]), S)
    assert np.array_equal(np.concatenate([p[1] for p in parts]), o)
    dd = synth.host_gdn(1, 70, Hk, Hv, d, d, seed=4, state_std=0.05)
    S2, o2 = orc.chunk_wy(dd["S0"], dd["q"], dd["k"], dd["v"], dd["g"], dd["beta"], scale=0.5, nthreads=1)
    assert np.array_equal(np.concatenate([h[0] for h in heads], axis=1), S2)
    assert np.array_equal(np.concatenate([h[1] for h in heads], axis=2), o2)
    assert tmax == 2.0
