"""orionsbelt_b200 -- B200 (sm_100a) Gated DeltaNet hot path behind the kai C ABI.

The product is libkai_gdn_cuda.so (C ABI: include/kai_gdn_cuda.h, CUDA
sources: csrc/).  This package builds it (``build``), binds it (``_lib``) and
mirrors the reference operator interface in Python (``ops``); ``synth``
makes the seeded synthetic inputs of the benchmark configurations.
"""
from ._lib import BF16, F16, F32, GdnError, LIB_PATH  # noqa: F401

__all__ = ["BF16", "F16", "F32", "GdnError", "LIB_PATH"]
