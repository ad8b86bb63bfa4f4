"""The allocation-free gated scan, kai_run_gdn_gated_scan_noalloc_sm100a.

It exists for callers that cannot allocate device memory at call time (an
engine that has given all of HBM to its own pools, or a host whose other
streams cannot wait for the device-wide synchronisation cudaMalloc/cudaFree
may bring); its segment carries live in a fixed array inside the library.

Checked through the C ABI against the existing entry point
kai_run_gdn_gated_scan_sm100a on the same inputs, on two calls in a row of
different shapes (the second call reuses the array the first one left
behind), with the tolerance the other gated-scan tests use
(gpu/gdn_gpu_validate.c:145 pass rule; in fact the results are identical).
This file sorts last so a run that stops at the first failure has already run
every other test; it also passes alone in a fresh process.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import validate_pass
from orionsbelt_b200 import _lib

pytestmark = pytest.mark.gpu


def _inputs(torch, batch, seq, ch, seed):
    r = np.random.default_rng(seed)
    g = torch.from_numpy(r.uniform(0.5, 0.99, (batch, seq, ch)).astype(np.float32)).cuda()
    x = torch.from_numpy(r.uniform(-1, 1, (batch, seq, ch)).astype(np.float32)).cuda()
    st = torch.from_numpy(r.uniform(-1, 1, (batch, ch)).astype(np.float32)).cuda()
    return g, x, st


def _call(fn, torch, g, x, st, batch, seq, ch):
    s = torch.full((batch, seq, ch), float("nan"), device="cuda")
    st = st.clone()
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(fn(g.data_ptr(), x.data_ptr(), s.data_ptr(), st.data_ptr(), _lib.F32, batch, seq, ch, stream))
    torch.cuda.synchronize()
    return s.cpu().numpy(), st.cpu().numpy()


@pytest.mark.parametrize("shapes", [[(2, 1000, 300), (1, 4096, 2048)]])
def test_noalloc_matches_existing_entry_point_twice(cuda, shapes):
    L = _lib.lib()
    for i, (batch, seq, ch) in enumerate(shapes):
        g, x, st = _inputs(cuda, batch, seq, ch, seed=100 + i)
        s_ref, st_ref = _call(L.kai_run_gdn_gated_scan_sm100a, cuda, g, x, st, batch, seq, ch)
        s_got, st_got = _call(L.kai_run_gdn_gated_scan_noalloc_sm100a, cuda, g, x, st, batch, seq, ch)
        assert not np.isnan(s_got).any()
        assert validate_pass(s_got, s_ref) and validate_pass(st_got, st_ref)
        assert np.array_equal(s_got, s_ref) and np.array_equal(st_got, st_ref)


def test_noalloc_rejects_calls_beyond_its_scratch(cuda):
    L = _lib.lib()
    batch, seq, ch = 1, 32768, 8192  # 2 * 256 * 8192 floats > the 4 MiB array
    g = cuda.empty((batch, seq, ch), device="cuda")
    s = cuda.empty_like(g)
    st = cuda.empty((batch, ch), device="cuda")
    rc = L.kai_run_gdn_gated_scan_noalloc_sm100a(g.data_ptr(), g.data_ptr(), s.data_ptr(), st.data_ptr(), _lib.F32,
                                                  batch, seq, ch, None)
    assert rc == _lib.ERR_INVALID
    assert "static maximum" in _lib.last_error()
    L.kai_gdn_cuda_clear_error()
