"""Reader / writer for the reference's tensor ``.bin`` format.

Test infrastructure only. Format (``scripts/verify_reference.py:30-65`` and
``tests/validation/src/tensor_compare.rs:79``): little-endian u32 ``ndim``,
``ndim`` u32 dims, u32 dtype enum (0 = float16, 1 = float32, 2 = int32), then
the raw row-major data.
"""

from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

_DTYPES = {0: np.float16, 1: np.float32, 2: np.int32}
_ENUMS = {np.dtype(np.float16): 0, np.dtype(np.float32): 1, np.dtype(np.int32): 2}


def load_tensor(path) -> np.ndarray:
    data = Path(path).read_bytes()
    (ndim,) = struct.unpack_from("<I", data, 0)
    shape = list(struct.unpack_from("<" + "I" * ndim, data, 4))
    (enum,) = struct.unpack_from("<I", data, 4 + 4 * ndim)
    if enum not in _DTYPES:
        raise ValueError(f"unknown dtype enum {enum} in {path}")
    off = 8 + 4 * ndim
    dt = np.dtype(_DTYPES[enum])
    n = int(np.prod(shape)) if shape else 0
    if len(data) - off != n * dt.itemsize:
        raise ValueError(f"size mismatch in {path}")
    return np.frombuffer(data, dtype=dt, count=n, offset=off).reshape(shape).copy()


def save_tensor(path, arr: np.ndarray) -> None:
    arr = np.ascontiguousarray(arr)
    enum = _ENUMS[arr.dtype]
    hdr = struct.pack("<I", arr.ndim) + struct.pack("<" + "I" * arr.ndim, *arr.shape) + struct.pack("<I", enum)
    Path(path).write_bytes(hdr + arr.tobytes())
