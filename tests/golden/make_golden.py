"""Generate the golden fixtures in tests/golden/ (run once, in a container that
has the reference tree and HF transformers; the .npz files are committed and
nothing at test time reads the reference tree).

  python tests/golden/make_golden.py [/path/to/reference]

Fixtures
  gdn1_recurrent.npz  bench/gdn2_reference.py::gdn1_recurrent (NumPy float64
                      token loop, the reference's own Python recurrence) on a
                      grouped-head case with a non-zero initial state.
  gdn2_uniform.npz    bench/gdn2_reference.py::gdn2_recurrent with uniform
                      erase/write gates (= GDN-1 with beta, the reduction
                      bench/gdn2_reference.py:293-351 tests), exercising the
                      reference's GDN-2 code path as a second anchor.
  gdn2_general.npz    bench/gdn2_reference.py::gdn2_recurrent with channel-wise
                      decay, erase and write gates (sigmoid / -softplus of
                      N(0,1), as its make_synthetic_input), grouped heads and a
                      non-zero initial state, d = 32: the GDN-2 decode step.
  hf_chunk.npz        HF transformers torch_chunk_gated_delta_rule (the chunkwise
                      WY form the reference reaches through bench/hf_backend.py)
                      on a multi-chunk case with a ragged last chunk.
  kai_lcg.npz         the reference's own C kernels (oracle/_ref/libgdnref.so) on
                      inputs from the LCG of kleidiai_submission/test_kai_gdn.c:45-51
                      (seed 0x5EED1234), at seq 64 x channels 33.
"""
from __future__ import annotations

import importlib
import importlib.util
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))


def lcg_fill(n: int, lo: float, hi: float, state: list) -> np.ndarray:
    """rand_float of kleidiai_submission/test_kai_gdn.c:45-51, in float32."""
    out = np.empty(n, np.float32)
    s = state[0]
    for i in range(n):
        s = (s * 1103515245 + 12345) & 0xFFFFFFFF
        r = np.float32((s >> 8) & 0xFFFFFF) / np.float32(0xFFFFFF)
        out[i] = np.float32(lo) + r * (np.float32(hi) - np.float32(lo))
    state[0] = s
    return out


def main(ref_root: Path, only=None) -> None:
    from orionsbelt_b200 import synth

    spec = importlib.util.spec_from_file_location("gdn2_reference", ref_root / "bench" / "gdn2_reference.py")
    G = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(G)

    # ---- gdn2_recurrent, general gates: T=5, Hk=2, Hv=4, K=V=32, S0 ~ N(0, 0.1)
    if only is None or "gdn2_general" in only:
        r = np.random.default_rng(14)
        T, Hk, Hv, K = 5, 2, 4, 32
        q = r.standard_normal((T, Hk, K)).astype(np.float32)
        k = r.standard_normal((T, Hk, K)).astype(np.float32)
        q /= np.linalg.norm(q, axis=-1, keepdims=True)
        k /= np.linalg.norm(k, axis=-1, keepdims=True)
        v = r.standard_normal((T, Hv, K)).astype(np.float32)
        g = (-np.log1p(np.exp(r.standard_normal((T, Hv, K))))).astype(np.float32)
        bg = (1.0 / (1.0 + np.exp(-r.standard_normal((T, Hv, K))))).astype(np.float32)
        wg = (1.0 / (1.0 + np.exp(-r.standard_normal((T, Hv, K))))).astype(np.float32)
        S0 = (0.1 * r.standard_normal((Hv, K, K))).astype(np.float32)
        scale = np.float32(1.0 / np.sqrt(K))
        og, Sg = G.gdn2_recurrent(q.astype(np.float64), k.astype(np.float64), v.astype(np.float64),
                                  g.astype(np.float64), bg.astype(np.float64), wg.astype(np.float64),
                                  scale=float(scale), initial_state=S0, use_qk_l2norm=False)
        np.savez_compressed(HERE / "gdn2_general.npz", q=q, k=k, v=v, g=g, b_gate=bg, w_gate=wg, S0=S0,
                            scale=scale, o=og, S=Sg)
        if only is not None:
            print("wrote gdn2_general.npz")
            return

    # ---- gdn1_recurrent: B=1, T=70, Hk=2, Hv=4, d=32, S0 ~ N(0, 0.1)
    d = synth.host_gdn(1, 70, 2, 4, 32, 32, g_scale=0.5, seed=11, state_std=0.1)
    scale = 1.0 / np.sqrt(32)
    qr = np.repeat(d["q"][0], 2, axis=1)
    kr = np.repeat(d["k"][0], 2, axis=1)
    o, S = G.gdn1_recurrent(qr, kr, d["v"][0], np.exp(d["g"][0].astype(np.float64)), d["beta"][0],
                            scale=scale, initial_state=d["S0"][0], use_qk_l2norm=False)
    np.savez_compressed(HERE / "gdn1_recurrent.npz", **d, scale=np.float32(scale), o=o, S=S)

    # ---- gdn2_recurrent with uniform gates: T=6, H=2, K=V=8
    d2 = synth.host_gdn(1, 6, 2, 2, 8, 8, g_scale=0.5, seed=12, state_std=0.0)
    T, H, K = 6, 2, 8
    g_ch = np.repeat(d2["g"][0][:, :, None], K, axis=2)          # log decay per channel
    b_gate = np.repeat(d2["beta"][0][:, :, None], K, axis=2)     # erase = beta
    w_gate = np.repeat(d2["beta"][0][:, :, None], K, axis=2)     # write = beta
    o2, S2 = G.gdn2_recurrent(d2["q"][0].astype(np.float64), d2["k"][0].astype(np.float64),
                              d2["v"][0].astype(np.float64), g_ch.astype(np.float64),
                              b_gate.astype(np.float64), w_gate.astype(np.float64), scale=1.0,
                              use_qk_l2norm=False)
    np.savez_compressed(HERE / "gdn2_uniform.npz", **d2, o=o2, S=S2)

    # ---- HF chunk: B=2, T=150 (3 chunks, ragged), Hk=2, Hv=4, d=32
    import torch
    from transformers.models.qwen3_5 import modeling_qwen3_5 as M

    d3 = synth.host_gdn(2, 150, 2, 4, 32, 32, g_scale=0.3, seed=13, state_std=0.05)
    q = torch.tensor(d3["q"]).repeat_interleave(2, dim=2)
    k = torch.tensor(d3["k"]).repeat_interleave(2, dim=2)
    oh, Sh = M.torch_chunk_gated_delta_rule(q, k, torch.tensor(d3["v"]), torch.tensor(d3["g"]),
                                            torch.tensor(d3["beta"]), chunk_size=64,
                                            initial_state=torch.tensor(d3["S0"]), output_final_state=True)
    np.savez_compressed(HERE / "hf_chunk.npz", **d3, scale=np.float32(1.0 / np.sqrt(32)),
                        o=oh.numpy(), S=Sh.numpy())

    # ---- reference C kernels on the kai test's LCG inputs
    import oracle

    oracle.build(ref=True)
    importlib.reload(oracle)
    ref = oracle.ref
    assert ref is not None, "reference library was not built"
    seq, ch = 64, 33
    st = [0x5EED1234]
    a = lcg_fill(seq * ch, 0.5, 1.5, st).reshape(seq, ch)
    g = lcg_fill(seq * ch, -0.99, 0.99, st).reshape(seq, ch)
    x = lcg_fill(seq * ch, -2.0, 2.0, st).reshape(seq, ch)
    s0 = lcg_fill(ch, -1.0, 1.0, st)
    cin = lcg_fill(seq * ch, -1.0, 1.0, st).reshape(seq, ch)
    w = lcg_fill(4 * ch, -1.0, 1.0, st).reshape(4, ch)
    h0 = lcg_fill(3 * ch, -1.0, 1.0, st).reshape(3, ch)
    ga = lcg_fill(128, -1.0, 1.0, st)
    gb = lcg_fill(128 * 33, -1.0, 1.0, st).reshape(128, 33)
    decay = ref.kai_cumdecay(a)
    s, s_state = ref.gated_scan(g, x, s0)
    conv_out, conv_hist = ref.conv(cin, w, h0)
    gemv = ref.gemv(ga, gb)
    np.savez_compressed(HERE / "kai_lcg.npz", a=a, decay=decay, g=g, x=x, s0=s0, s=s, s_state=s_state,
                        cin=cin, w=w, h0=h0, conv_out=conv_out, conv_hist=conv_hist, ga=ga, gb=gb, gemv=gemv)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    # python make_golden.py [reference root] [fixture names to (re)write only]
    # (the root defaults to the ORIONSBELT_REF environment variable)
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("ORIONSBELT_REF")
    if not root:
        sys.exit("usage: make_golden.py <reference root> [names]  (or set ORIONSBELT_REF)")
    main(Path(root), set(sys.argv[2:]) or None)
