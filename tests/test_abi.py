"""CPU checks of the C-ABI library: it loads, exports every declared symbol, and
its host-side pieces (tables, argument checks) behave — no GPU needed."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

from fracture_b200 import _lib, kernels as K
from oracle import ops, turboquant as tq

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "fracture_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", text, flags=re.M))
                  - {"if", "sizeof"})


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    names = declared_functions()
    assert len(names) >= 50, names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # the Python binding declares exactly the header's functions
    assert sorted(_lib.SIGNATURES) == names


def test_reference_abi_symbols_present():
    """The seven kernels Fracture's FFI binds (backends/fracture-cuda/src/ffi.rs:141-249)."""
    lib = _lib.load()
    for n in ["launch_rmsnorm", "launch_rope", "launch_silu_mul", "launch_embedding", "launch_add",
              "launch_turboquant_compress", "launch_turboquant_decompress"]:
        assert hasattr(lib, n)


def test_rope_tables_bit_exact():
    for hd, theta in [(128, 500000.0), (32, 500000.0), (64, 10000.0)]:
        assert np.array_equal(K.rope_freqs(hd, theta), ops.rope_freqs(hd, theta))
    assert np.array_equal(K.rope_freqs_llama3(128, 5e5, 8.0, 1.0, 4.0, 8192),
                          ops.rope_freqs_llama3(128, 5e5, 8.0, 1.0, 4.0, 8192))


@pytest.mark.parametrize("dim,bits", [(128, 2), (128, 3), (128, 4), (16, 4), (32, 2), (64, 4)])
def test_codebook_bit_exact(dim, bits):
    c, b = K.tq_codebook(dim, bits)
    cb = tq.get_codebook(dim, bits)
    assert np.array_equal(c, cb.centroids) and np.array_equal(b, cb.boundaries)


@pytest.mark.parametrize("d,seed", [(16, 42), (32, 43), (128, 42), (128, 542), (128, 31042)])
def test_rotation_bit_exact(d, seed):
    assert np.array_equal(K.tq_rotation_matrix(d, seed), tq.generate_rotation_matrix(d, seed))


def test_argument_checks_reject_before_launch():
    """Rejected arguments return cudaErrorInvalidValue (1) before anything is enqueued."""
    lib = _lib.load()
    assert lib.launch_add(None, None, None, -1, None) == 1
    assert lib.launch_silu_mul(None, None, None, -5, None) == 1
    assert lib.fb_launch_add(None, None, None, 10, 0, None) == 1          # null pointers
    assert lib.fb_launch_rmsnorm(None, None, None, 1e-5, 4, 8, 7, None) == 1  # bad dtype -> also null
    assert lib.fb_launch_rope(None, None, None, None, 4, 2, 1, 7, 0, None) == 1  # odd head_dim
    # TurboQuant: bit widths and packed dims are checked as the reference config does
    assert lib.launch_turboquant_compress(None, None, None, None, None, 1, 1, 128, 32, 5, 80, None) == 1
    assert lib.launch_turboquant_compress(None, None, None, None, None, 1, 1, 128, 16, 4, 63, None) == 1
    assert lib.launch_turboquant_compress(None, None, None, None, None, 1, 1, 128, 8, 4, 64, None) == 1
    assert lib.launch_turboquant_decompress(None, None, None, None, None, 1, 1, 128, 6, 96, None) == 1
    assert lib.fb_launch_tq_compress_paged(None, 0, None, None, 4, 4, 8, 256, None, 0, 16, None, None, None, None) == 1
    # K+V in one call: a slot map is required when there are tokens; widths are checked per side
    kv = lambda kb, vb, n, slots: lib.fb_launch_tq_compress_kv_slots(None, None, 0, None, None, None, None, kb, vb,
                                                                     n, 8, 128, slots, 16, None, None, None, None,
                                                                     None, None)
    assert kv(4, 4, 4, None) == 1
    assert kv(4, 5, 4, None) == 1
    assert kv(4, 2, 0, None) == 0  # empty: nothing to do
    assert kv(5, 4, 0, None) == 1  # a bad width is rejected even when empty
    assert lib.fb_launch_tq_compress_kv_paged(None, None, 0, None, None, None, None, 4, 4, 4, 8, 128, None, 0, 16,
                                              None, None, None, None, None, None) == 1
    # empty inputs are a no-op success
    assert lib.launch_add(None, None, None, 0, None) == 0
    assert lib.fb_launch_tq_compress_paged(None, 0, None, None, 4, 0, 8, 128, None, 0, 0, None, None, None, None) == 0


def test_path_counters_match_the_python_names():
    """fb_tq_path_counts fills exactly one counter per name in kernels.TQ_PATHS (a host call, no GPU)."""
    import ctypes as C

    lib = _lib.load()
    n = len(K.TQ_PATHS)
    arr = (C.c_ulonglong * (n + 4))(*([0xDEAD] * (n + 4)))
    assert lib.fb_tq_path_counts(arr, n + 4) == 0
    assert all(v != 0xDEAD for v in arr[:n]) and all(v == 0xDEAD for v in arr[n:])
    assert lib.fb_tq_path_counts(None, n) == 1


def test_invalid_table_arguments():
    lib = _lib.load()
    out = np.zeros(64, dtype=np.float32)
    assert lib.fb_rope_freqs(127, 5e5, out.ctypes.data_as(_lib.f32p)) != 0
    assert lib.fb_rope_freqs_llama3(128, 5e5, 8.0, 4.0, 1.0, 8192.0, out.ctypes.data_as(_lib.f32p)) != 0
    assert lib.fb_tq_codebook(128, 9, None, None) != 0
