"""ctypes binding of ``libfracture_b200.so`` (declarations mirror ``include/fracture_b200.h``).

The library is built in-tree by ``fracture_b200.build``. Loading fails loudly
when it is missing: there is no fallback implementation.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libfracture_b200.so"

FB_FP16, FB_FP32, FB_BF16, FB_INT8, FB_INT4 = 0, 1, 2, 3, 4

vp = C.c_void_p
i32 = C.c_int
i64 = C.c_int64
u32p = C.POINTER(C.c_uint32)
f32p = C.POINTER(C.c_float)
szt = C.c_size_t


class FbTensor(C.Structure):
    _fields_ = [("id", C.c_uint64), ("dtype", C.c_int32), ("ndim", C.c_int32), ("shape", C.c_int64 * 4)]


class FbTqConfig(C.Structure):
    _fields_ = [("key_bits", C.c_uint8), ("value_bits", C.c_uint8), ("protected_bits", C.c_uint8),
                ("pad0", C.c_uint8), ("protected_layers", C.c_uint32), ("residual_tokens", C.c_uint32),
                ("seed", C.c_uint64)]


class FbRopeParams(C.Structure):
    _fields_ = [("theta", C.c_double), ("factor", C.c_double), ("original_context", C.c_double),
                ("low_freq_factor", C.c_double), ("high_freq_factor", C.c_double), ("scaling", C.c_int32),
                ("head_dim", C.c_int32), ("num_freq_factors", C.c_int32), ("pad0", C.c_int32)]


FB_ROPE_SCALING = {0: "none", 1: "linear", 2: "llama3", 3: "factors"}

TP = C.POINTER(FbTensor)

# name -> (restype, argtypes)
SIGNATURES = {
    # 1. reference kernel ABI
    "launch_rmsnorm": (i32, [vp, vp, vp, C.c_float, i32, i32, vp]),
    "launch_rope": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, vp]),
    "launch_silu_mul": (i32, [vp, vp, vp, i32, vp]),
    "launch_embedding": (i32, [vp, vp, vp, i32, i32, i32, vp]),
    "launch_add": (i32, [vp, vp, vp, i32, vp]),
    "launch_turboquant_compress": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp]),
    "launch_turboquant_decompress": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]),
    "launch_attention_paged_tq": (i32, [vp] * 11 + [i32] * 10 + [vp]),
    "launch_attention_paged_tq_noalloc": (i32, [vp] * 11 + [i32] * 10 + [vp]),
    "launch_paged_attention": (i32, [vp] * 5 + [i32] * 7 + [vp]),
    # 2. new kernel entry points
    "fb_launch_embedding": (i32, [vp, vp, vp, i64, i64, i64, i32, vp]),
    "fb_launch_add": (i32, [vp, vp, vp, i64, i32, vp]),
    "fb_launch_rmsnorm": (i32, [vp, vp, vp, C.c_float, i64, i64, i32, vp]),
    "fb_launch_add_rmsnorm": (i32, [vp, vp, vp, vp, C.c_float, i64, i64, i32, vp]),
    "fb_launch_rope": (i32, [vp, vp, vp, vp, i64, i32, i32, i32, i32, vp]),
    "fb_launch_silu_mul": (i32, [vp, vp, vp, i64, i32, vp]),
    "fb_launch_tq_compress_paged": (i32, [vp, i32, vp, vp, i32, i64, i32, i32, vp, i64, i64, vp, vp, vp, vp]),
    "fb_launch_tq_compress_kv_paged": (i32, [vp, vp, i32, vp, vp, vp, vp, i32, i32, i64, i32, i32, vp, i64, i64,
                                             vp, vp, vp, vp, vp, vp]),
    "fb_launch_tq_dequant_kv_paged": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i64, i32, i32, vp, i64, i64,
                                            vp, vp, i32, vp]),
    "fb_launch_tq_dequant_paged": (i32, [vp, vp, vp, vp, i32, i64, i32, i32, vp, i64, i64, vp, i32, vp]),
    "fb_launch_tq_compress_slots": (i32, [vp, i32, vp, vp, i32, i64, i32, i32, vp, i64, vp, vp, vp, vp]),
    "fb_launch_tq_compress_kv_slots": (i32, [vp, vp, i32, vp, vp, vp, vp, i32, i32, i64, i32, i32, vp, i64,
                                             vp, vp, vp, vp, vp, vp]),
    "fb_launch_tq_dequant_slots": (i32, [vp, vp, vp, vp, i32, i64, i32, i32, vp, i64, vp, i32, vp]),
    "fb_tq_attention_workspace_bytes": (C.c_size_t, [i32, i32, i32, i32]),
    "fb_launch_tq_attention_paged": (i32, [vp, i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, i64, vp, i32, vp, vp,
                                           i32, vp, vp, vp, vp, i32, i32, vp, C.c_size_t, vp, vp]),
    "fb_attention_workspace_bytes": (C.c_size_t, [i32, i32, i32, i32]),
    "fb_launch_attention_paged": (i32, [vp, i32, i32, i32, i32, i32, i32, vp, vp, i64, vp, i32, vp, vp, i32, vp,
                                        C.c_size_t, vp, vp]),
    "fb_launch_kv_append_paged": (i32, [vp, vp, i32, i64, i32, i32, vp, i64, i64, vp, vp, vp, vp]),
    "fb_tq_timeouts": (C.c_uint, []),
    "fb_tq_path_counts": (i32, [C.POINTER(C.c_ulonglong), i32]),
    "fb_rope_freqs": (i32, [i32, C.c_double, f32p]),
    "fb_rope_freqs_llama3": (i32, [i32, C.c_double, C.c_double, C.c_double, C.c_double, C.c_double, f32p]),
    "fb_tq_codebook": (i32, [i32, i32, f32p, f32p]),
    "fb_tq_rotation_matrix": (i32, [i32, C.c_uint64, f32p]),
    "fb_gguf_rope_params": (i32, [C.c_char_p, C.POINTER(FbRopeParams)]),
    "fb_rope_freqs_from_gguf": (i32, [C.c_char_p, i32, f32p]),
    "fb_gguf_last_error": (C.c_char_p, []),
    # 3. backend object
    "fb_last_error": (C.c_char_p, []),
    "fb_backend_create": (i32, [i32, C.POINTER(vp)]),
    "fb_backend_destroy": (i32, [vp]),
    "fb_backend_stream": (i32, [vp, C.POINTER(vp)]),
    "fb_backend_device_name": (i32, [vp, C.c_char_p, szt]),
    "fb_backend_total_memory": (i32, [vp, C.POINTER(szt)]),
    "fb_backend_available_memory": (i32, [vp, C.POINTER(szt)]),
    "fb_alloc": (i32, [vp, C.POINTER(C.c_int64), i32, i32, TP]),
    "fb_free": (i32, [vp, TP]),
    "fb_copy_to_device": (i32, [vp, TP, vp, szt]),
    "fb_copy_to_host": (i32, [vp, TP, vp, szt]),
    "fb_register_external": (i32, [vp, vp, C.POINTER(C.c_int64), i32, i32, TP]),
    "fb_get_ptr": (i32, [vp, TP, C.POINTER(vp)]),
    "fb_rmsnorm": (i32, [vp, TP, TP, C.c_double, TP]),
    "fb_rope": (i32, [vp, TP, TP, u32p, szt, C.c_double, szt]),
    "fb_silu_mul": (i32, [vp, TP, TP, TP]),
    "fb_embedding": (i32, [vp, u32p, szt, TP, TP]),
    "fb_add": (i32, [vp, TP, TP, TP]),
    "fb_copy_rows": (i32, [vp, TP, TP, szt, szt, szt]),
    "fb_turboquant_compress": (i32, [vp, TP, TP, TP, C.c_uint8, TP, TP]),
    "fb_synchronize": (i32, [vp]),
    "fb_precompute_rope_freqs": (i32, [vp, szt, C.c_double]),
    "fb_precompute_rope_freqs_llama3": (i32, [vp, szt, C.c_double, C.c_double, C.c_double, C.c_double, C.c_double]),
    "fb_precompute_rope_freqs_gguf": (i32, [vp, szt, C.c_char_p]),
    "fb_create_timer": (i32, [vp, C.POINTER(C.c_uint64)]),
    "fb_start_timer": (i32, [vp, C.c_uint64]),
    "fb_stop_timer": (i32, [vp, C.c_uint64, C.POINTER(C.c_float)]),
    "fb_destroy_timer": (i32, [vp, C.c_uint64]),
    "fb_tq_cache_create": (i32, [vp, szt, szt, szt, szt, C.POINTER(FbTqConfig), C.POINTER(vp)]),
    "fb_tq_cache_destroy": (i32, [vp]),
    "fb_tq_cache_alloc": (i32, [vp, C.POINTER(C.c_uint64)]),
    "fb_tq_cache_free": (i32, [vp, C.c_uint64]),
    "fb_tq_cache_append_kv": (i32, [vp, C.c_uint64, szt, TP, TP]),
    "fb_tq_cache_block_table": (i32, [vp, C.c_uint64, C.POINTER(C.c_int32), szt, C.POINTER(szt)]),
    "fb_tq_cache_seq_len": (i32, [vp, C.c_uint64, C.POINTER(szt)]),
    "fb_tq_cache_num_free_blocks": (i32, [vp, C.POINTER(szt)]),
    "fb_tq_cache_pool": (i32, [vp, szt, i32, C.POINTER(vp), C.POINTER(vp), C.POINTER(vp), C.POINTER(vp),
                                C.POINTER(i32)]),
    "fb_tq_cache_dequant": (i32, [vp, C.c_uint64, szt, i32, szt, TP]),
    "fb_tq_cache_attention": (i32, [vp, C.c_uint64, szt, TP, szt, szt, TP]),
    "fb_kv_cache_create": (i32, [vp, szt, szt, szt, szt, i32, C.POINTER(vp)]),
    "fb_kv_cache_destroy": (i32, [vp]),
    "fb_kv_cache_alloc": (i32, [vp, C.POINTER(C.c_uint64)]),
    "fb_kv_cache_free": (i32, [vp, C.c_uint64]),
    "fb_kv_cache_append_kv": (i32, [vp, C.c_uint64, szt, TP, TP]),
    "fb_kv_cache_block_table": (i32, [vp, C.c_uint64, C.POINTER(C.c_int32), szt, C.POINTER(szt)]),
    "fb_kv_cache_seq_len": (i32, [vp, C.c_uint64, C.POINTER(szt), C.POINTER(szt)]),
    "fb_kv_cache_num_free_blocks": (i32, [vp, C.POINTER(szt)]),
    "fb_kv_cache_pool": (i32, [vp, szt, C.POINTER(vp), C.POINTER(vp)]),
    "fb_kv_cache_attention": (i32, [vp, C.c_uint64, szt, TP, szt, szt, TP]),
}

_LIB = None


def load() -> C.CDLL:
    """Load the in-tree library (raises if it has not been built)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} not built: run `python -m fracture_b200.build` "
                          "(the CUDA library is required; there is no fallback)")
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib
