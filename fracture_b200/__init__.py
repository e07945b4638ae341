"""fracture_b200 — B200-native (sm_100a) kernels for Fracture's per-layer
elementwise hot path and TurboQuant KV compression.

The product is the C-ABI library ``libfracture_b200.so`` (see
``include/fracture_b200.h``); this package builds it (``build``), binds it
(``_lib``), exposes the reference's ``Backend`` trait over it (``backend``)
and torch-facing wrappers of the raw launches (``kernels``).
"""

from ._lib import FB_BF16, FB_FP16, FB_FP32, FB_INT4, FB_INT8, LIB_PATH, load  # noqa: F401

__all__ = ["load", "LIB_PATH", "FB_FP16", "FB_FP32", "FB_BF16", "FB_INT8", "FB_INT4"]
