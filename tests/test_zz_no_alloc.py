"""The allocation-free gated scan, kai_run_gdn_gated_scan_noalloc_sm100a.

It exists for callers that cannot allocate device memory at call time (an
engine that has given all of HBM to its own pools, or a host whose other
streams cannot wait for the device-wide synchronisation cudaMalloc/cudaFree
may bring); its segment carries live in a fixed array inside the library.

Checked through the C ABI against the existing entry point
kai_run_gdn_gated_scan_sm100a on the same inputs, on two calls in a row of
different shapes (the second call reuses the array the first one left
behind), for fp32, fp16 and bf16 state, with the tolerance the other
gated-scan tests use (gpu/gdn_gpu_validate.c:145 pass rule; in fact the
results are identical).  Also: a call on a stream the library has never seen
leaves the device's free memory unchanged, the largest call the array holds
runs, and the next size up is refused.  This file sorts last so a run that
stops at the first failure has already run every other test; it also passes
alone in a fresh process.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import validate_pass
from orionsbelt_b200 import _lib

pytestmark = pytest.mark.gpu

_DT = {"f32": (_lib.F32, "float32"), "f16": (_lib.F16, "float16"), "bf16": (_lib.BF16, "bfloat16")}


def _inputs(torch, batch, seq, ch, seed, sdt="f32"):
    r = np.random.default_rng(seed)
    g = torch.from_numpy(r.uniform(0.5, 0.99, (batch, seq, ch)).astype(np.float32)).cuda()
    x = torch.from_numpy(r.uniform(-1, 1, (batch, seq, ch)).astype(np.float32)).cuda()
    st = torch.from_numpy(r.uniform(-1, 1, (batch, ch)).astype(np.float32)).cuda().to(getattr(torch, _DT[sdt][1]))
    return g, x, st


def _call(fn, torch, g, x, st, batch, seq, ch, sdt="f32", stream=None):
    s = torch.full((batch, seq, ch), float("nan"), device="cuda")
    st = st.clone()
    sp = (stream or torch.cuda.current_stream()).cuda_stream
    _lib.check(fn(g.data_ptr(), x.data_ptr(), s.data_ptr(), st.data_ptr(), _DT[sdt][0], batch, seq, ch, sp))
    torch.cuda.synchronize()
    return s.cpu().numpy(), st.float().cpu().numpy()


# Tile records: 256 + 512 * batch * ceil(seq / 256) * ceil(channels / 32)
# bytes, at most KAI_GDN_NOALLOC_SCRATCH_BYTES (4 MiB): 8191 tiles at most.
def _need(batch, seq, ch):
    return 256 + 512 * batch * (-(-seq // 256)) * (-(-ch // 32))


@pytest.mark.parametrize("sdt", ["f32", "f16", "bf16"])
def test_noalloc_matches_existing_entry_point_twice(cuda, sdt):
    L = _lib.lib()
    for i, (batch, seq, ch) in enumerate([(2, 1000, 300), (1, 4096, 2048)]):
        g, x, st = _inputs(cuda, batch, seq, ch, seed=100 + i, sdt=sdt)
        s_ref, st_ref = _call(L.kai_run_gdn_gated_scan_sm100a, cuda, g, x, st, batch, seq, ch, sdt)
        s_got, st_got = _call(L.kai_run_gdn_gated_scan_noalloc_sm100a, cuda, g, x, st, batch, seq, ch, sdt)
        assert not np.isnan(s_got).any()
        assert validate_pass(s_got, s_ref) and validate_pass(st_got, st_ref)
        assert np.array_equal(s_got, s_ref) and np.array_equal(st_got, st_ref)


def test_noalloc_allocates_nothing_on_a_new_stream(cuda):
    L = _lib.lib()
    batch, seq, ch = 1, 4096, 2048
    g, x, st = _inputs(cuda, batch, seq, ch, seed=7)
    s = cuda.empty((batch, seq, ch), device="cuda")
    _call(L.kai_run_gdn_gated_scan_noalloc_sm100a, cuda, g, x, st, batch, seq, ch)  # loads the module
    fresh = cuda.cuda.Stream()
    cuda.cuda.synchronize()
    free0, _ = cuda.cuda.mem_get_info()
    _lib.check(L.kai_run_gdn_gated_scan_noalloc_sm100a(g.data_ptr(), x.data_ptr(), s.data_ptr(), st.data_ptr(),
                                                       _lib.F32, batch, seq, ch, fresh.cuda_stream))
    fresh.synchronize()
    free1, _ = cuda.cuda.mem_get_info()
    assert free1 == free0


def test_noalloc_largest_call_runs_and_next_size_is_refused(cuda):
    L = _lib.lib()
    limit = 4 << 20
    batch, ch = 1, 32
    seq = 256 * 8191
    assert _need(batch, seq, ch) <= limit < _need(batch, seq + 256, ch)
    g, x, st = _inputs(cuda, batch, seq, ch, seed=9)
    s_ref, st_ref = _call(L.kai_run_gdn_gated_scan_sm100a, cuda, g, x, st, batch, seq, ch)
    s_got, st_got = _call(L.kai_run_gdn_gated_scan_noalloc_sm100a, cuda, g, x, st, batch, seq, ch)
    assert np.array_equal(s_got, s_ref) and np.array_equal(st_got, st_ref)
    del s_ref, s_got
    big = seq + 256  # one tile more than the array holds
    gb = cuda.empty((batch, big, ch), device="cuda")
    sb = cuda.empty_like(gb)
    rc = L.kai_run_gdn_gated_scan_noalloc_sm100a(gb.data_ptr(), gb.data_ptr(), sb.data_ptr(), st.data_ptr(),
                                                  _lib.F32, batch, big, ch, None)
    assert rc == _lib.ERR_INVALID
    assert "static maximum" in _lib.last_error()
    L.kai_gdn_cuda_clear_error()


def test_noalloc_rejects_calls_beyond_its_scratch(cuda):
    L = _lib.lib()
    batch, seq, ch = 1, 32768, 8192  # 256 + 512 * 128 * 256 bytes = 16.8 MB > the 4 MiB array
    assert _need(batch, seq, ch) > 4 << 20
    g = cuda.empty((batch, seq, ch), device="cuda")
    s = cuda.empty_like(g)
    st = cuda.empty((batch, ch), device="cuda")
    rc = L.kai_run_gdn_gated_scan_noalloc_sm100a(g.data_ptr(), g.data_ptr(), s.data_ptr(), st.data_ptr(), _lib.F32,
                                                  batch, seq, ch, None)
    assert rc == _lib.ERR_INVALID
    assert "static maximum" in _lib.last_error()
    L.kai_gdn_cuda_clear_error()
