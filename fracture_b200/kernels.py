"""torch-facing wrappers of the raw kernel entry points (layers 1-2 of the C ABI).

torch is used only for device memory and the current stream; every launch
goes through ``libfracture_b200.so``. Each wrapper checks the returned
cudaError_t and raises ``RuntimeError`` on failure.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from ._lib import FB_BF16, FB_FP16, FB_FP32

TORCH_DT = {torch.float16: FB_FP16, torch.bfloat16: FB_BF16, torch.float32: FB_FP32}


def _stream(stream=None) -> int:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return stream if isinstance(stream, int) else stream.cuda_stream


def _ok(rc: int, name: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{name} failed: cudaError {rc}")


def _dt(t: torch.Tensor) -> int:
    return TORCH_DT[t.dtype]


def silu_mul(out, gate, up, stream=None):
    _ok(_lib.load().fb_launch_silu_mul(out.data_ptr(), gate.data_ptr(), up.data_ptr(), gate.numel(), _dt(gate),
                                       _stream(stream)), "silu_mul")


def add(out, a, b, stream=None):
    _ok(_lib.load().fb_launch_add(out.data_ptr(), a.data_ptr(), b.data_ptr(), a.numel(), _dt(a), _stream(stream)), "add")


def rmsnorm(out, x, w, eps, stream=None):
    rows, cols = x.shape[0], x.shape[-1]
    _ok(_lib.load().fb_launch_rmsnorm(out.data_ptr(), x.data_ptr(), w.data_ptr(), float(eps), rows, cols, _dt(x),
                                      _stream(stream)), "rmsnorm")


def add_rmsnorm(h, residual, w, normed, eps, stream=None):
    rows, cols = h.shape[0], h.shape[-1]
    _ok(_lib.load().fb_launch_add_rmsnorm(h.data_ptr(), residual.data_ptr(), w.data_ptr(), normed.data_ptr(),
                                          float(eps), rows, cols, _dt(h), _stream(stream)), "add_rmsnorm")


def embedding(out, table, ids, stream=None):
    _ok(_lib.load().fb_launch_embedding(out.data_ptr(), table.data_ptr(), ids.data_ptr(), ids.numel(),
                                        table.shape[1], table.shape[0], _dt(table), _stream(stream)), "embedding")


def rope(q, k, positions, freqs, stream=None):
    T, nq, hd = q.shape
    nkv = k.shape[1]
    _ok(_lib.load().fb_launch_rope(q.data_ptr(), k.data_ptr(), positions.data_ptr(), freqs.data_ptr(), T, nq, nkv,
                                   hd, _dt(q), _stream(stream)), "rope")


def tq_compress_paged(x, rotation, centroids, bits, packed_pool, norms_pool, block_table=None, start_pos=0,
                      err=None, stream=None):
    T, H, d = x.shape
    rows = norms_pool.shape[0]
    _ok(_lib.load().fb_launch_tq_compress_paged(
        x.data_ptr(), _dt(x), rotation.data_ptr(), centroids.data_ptr(), bits, T, H, d,
        block_table.data_ptr() if block_table is not None else None, start_pos, rows, packed_pool.data_ptr(),
        norms_pool.data_ptr(), err.data_ptr() if err is not None else None, _stream(stream)), "tq_compress_paged")


def tq_compress_kv_paged(k, v, k_rotation, v_rotation, k_centroids, v_centroids, key_bits, value_bits, k_pool,
                         k_norms, v_pool, v_norms, block_table=None, start_pos=0, err=None, stream=None):
    """K and V of one append (``[T, H, d]`` each) into their pools, one launch where both qualify."""
    T, H, d = k.shape
    assert v.shape == k.shape and v.dtype == k.dtype and v_norms.shape[0] == k_norms.shape[0]
    rows = k_norms.shape[0]
    _ok(_lib.load().fb_launch_tq_compress_kv_paged(
        k.data_ptr(), v.data_ptr(), _dt(k), k_rotation.data_ptr(), v_rotation.data_ptr(), k_centroids.data_ptr(),
        v_centroids.data_ptr(), key_bits, value_bits, T, H, d,
        block_table.data_ptr() if block_table is not None else None, start_pos, rows, k_pool.data_ptr(),
        k_norms.data_ptr(), v_pool.data_ptr(), v_norms.data_ptr(), err.data_ptr() if err is not None else None,
        _stream(stream)), "tq_compress_kv_paged")


def tq_dequant_paged(packed_pool, norms_pool, rotation, centroids, bits, out, block_table=None, start_pos=0,
                     stream=None):
    T, H, d = out.shape
    rows = norms_pool.shape[0]
    _ok(_lib.load().fb_launch_tq_dequant_paged(
        packed_pool.data_ptr(), norms_pool.data_ptr(), rotation.data_ptr(), centroids.data_ptr(), bits, T, H, d,
        block_table.data_ptr() if block_table is not None else None, start_pos, rows, out.data_ptr(), _dt(out),
        _stream(stream)), "tq_dequant_paged")


def tq_dequant_kv_paged(k_pool, k_norms, v_pool, v_norms, k_rotation, v_rotation, k_centroids, v_centroids,
                        key_bits, value_bits, k_out, v_out, block_table=None, start_pos=0, stream=None):
    """K and V of one cache read into ``k_out``/``v_out`` (``[T, H, d]``), one launch where both qualify."""
    T, H, d = k_out.shape
    assert v_out.shape == k_out.shape and v_out.dtype == k_out.dtype
    rows = k_norms.shape[0]
    _ok(_lib.load().fb_launch_tq_dequant_kv_paged(
        k_pool.data_ptr(), k_norms.data_ptr(), v_pool.data_ptr(), v_norms.data_ptr(), k_rotation.data_ptr(),
        v_rotation.data_ptr(), k_centroids.data_ptr(), v_centroids.data_ptr(), key_bits, value_bits, T, H, d,
        block_table.data_ptr() if block_table is not None else None, start_pos, rows, k_out.data_ptr(),
        v_out.data_ptr(), _dt(k_out), _stream(stream)), "tq_dequant_kv_paged")


def tq_compress_slots(x, rotation, centroids, bits, packed_pool, norms_pool, slot_map, err=None, stream=None):
    """Batched append: token t of ``x [T, H, d]`` into pool row ``slot_map[t]`` (int64 tensor)."""
    T, H, d = x.shape
    rows = norms_pool.shape[0]
    _ok(_lib.load().fb_launch_tq_compress_slots(
        x.data_ptr(), _dt(x), rotation.data_ptr(), centroids.data_ptr(), bits, T, H, d, slot_map.data_ptr(), rows,
        packed_pool.data_ptr(), norms_pool.data_ptr(), err.data_ptr() if err is not None else None, _stream(stream)),
        "tq_compress_slots")


def tq_compress_kv_slots(k, v, k_rotation, v_rotation, k_centroids, v_centroids, key_bits, value_bits, k_pool,
                         k_norms, v_pool, v_norms, slot_map, err=None, stream=None):
    """K and V of one batched append (``[T, H, d]`` each) through one slot map, one launch where both qualify."""
    T, H, d = k.shape
    assert v.shape == k.shape and v.dtype == k.dtype and v_norms.shape[0] == k_norms.shape[0]
    rows = k_norms.shape[0]
    _ok(_lib.load().fb_launch_tq_compress_kv_slots(
        k.data_ptr(), v.data_ptr(), _dt(k), k_rotation.data_ptr(), v_rotation.data_ptr(), k_centroids.data_ptr(),
        v_centroids.data_ptr(), key_bits, value_bits, T, H, d, slot_map.data_ptr(), rows, k_pool.data_ptr(),
        k_norms.data_ptr(), v_pool.data_ptr(), v_norms.data_ptr(), err.data_ptr() if err is not None else None,
        _stream(stream)), "tq_compress_kv_slots")


def tq_dequant_slots(packed_pool, norms_pool, rotation, centroids, bits, out, slot_map, stream=None):
    """Gather: ``out[t]`` dequantized from pool row ``slot_map[t]`` (int64 tensor)."""
    T, H, d = out.shape
    rows = norms_pool.shape[0]
    _ok(_lib.load().fb_launch_tq_dequant_slots(
        packed_pool.data_ptr(), norms_pool.data_ptr(), rotation.data_ptr(), centroids.data_ptr(), bits, T, H, d,
        slot_map.data_ptr(), rows, out.data_ptr(), _dt(out), _stream(stream)), "tq_dequant_slots")


TQ_PATHS = ("compress_small", "compress_tensor_core", "compress_exact", "dequant_small", "dequant_tensor_core",
            "dequant_exact", "compress_kv_fused", "dequant_kv_fused", "attention_cuda_core", "attention_per_head",
            "attention_streamed", "compress_kv_small")


def tq_path_counts() -> dict:
    """Calls served so far by each TurboQuant kernel family (fb_tq_path_counts)."""
    arr = (C.c_ulonglong * len(TQ_PATHS))()
    _ok(_lib.load().fb_tq_path_counts(arr, len(TQ_PATHS)), "fb_tq_path_counts")
    return dict(zip(TQ_PATHS, (int(v) for v in arr)))


def tq_attention_workspace_bytes(num_seqs, q_per_seq, num_q_heads, max_kv_len) -> int:
    return int(_lib.load().fb_tq_attention_workspace_bytes(num_seqs, q_per_seq, num_q_heads, max_kv_len))


def tq_attention_paged(q, k_pool, k_norms, v_pool, v_norms, block_tables, kv_lens, start_pos, k_rotation,
                       v_rotation, k_centroids, v_centroids, key_bits, value_bits, out, max_kv_len=None,
                       workspace=None, stream=None):
    """Attention of ``q [S, Tq, Hq, 128]`` over the compressed paged cache of S sequences.

    ``block_tables [S, max_blocks]`` int32, ``kv_lens`` / ``start_pos`` ``[S]`` int32 (device);
    pools as ``tq_compress_paged`` writes them (``[rows, Hkv * P]`` uint8, norms ``[rows, Hkv]``
    fp16). ``out`` like ``q``. A workspace is allocated when none is given."""
    S, Tq, Hq, d = q.shape
    Hkv = k_norms.shape[1]
    if max_kv_len is None:
        max_kv_len = int(kv_lens.max().item()) if kv_lens.numel() else 0
    need = tq_attention_workspace_bytes(S, Tq, Hq, max_kv_len)
    if workspace is None:
        workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=q.device)
    _ok(_lib.load().fb_launch_tq_attention_paged(
        q.data_ptr(), _dt(q), S, Tq, Hq, Hkv, d, k_pool.data_ptr(), k_norms.data_ptr(), v_pool.data_ptr(),
        v_norms.data_ptr(), k_norms.shape[0], block_tables.data_ptr(), block_tables.shape[1], kv_lens.data_ptr(),
        start_pos.data_ptr(), max_kv_len, k_rotation.data_ptr(), v_rotation.data_ptr(), k_centroids.data_ptr(),
        v_centroids.data_ptr(), key_bits, value_bits, workspace.data_ptr(), workspace.numel(), out.data_ptr(),
        _stream(stream)), "tq_attention_paged")


def kv_append_paged(keys, values, k_pool, v_pool, block_table, start_pos=0, err=None, stream=None):
    """Write ``keys``/``values [T, Hkv, d]`` into the pools ``[rows, Hkv, d]`` through the block table."""
    T, H, d = keys.shape
    _ok(_lib.load().fb_launch_kv_append_paged(
        keys.data_ptr(), values.data_ptr(), _dt(keys), T, H, d, block_table.data_ptr(), start_pos, k_pool.shape[0],
        k_pool.data_ptr(), v_pool.data_ptr(), err.data_ptr() if err is not None else None, _stream(stream)),
        "kv_append_paged")


def attention_workspace_bytes(num_seqs, q_per_seq, num_q_heads, max_kv_len) -> int:
    return int(_lib.load().fb_attention_workspace_bytes(num_seqs, q_per_seq, num_q_heads, max_kv_len))


def attention_paged(q, k_pool, v_pool, block_tables, kv_lens, start_pos, out, max_kv_len=None, workspace=None,
                    stream=None):
    """Attention of ``q [S, Tq, Hq, 128]`` over the FP16/BF16 paged cache (pools ``[rows, Hkv, 128]``)."""
    S, Tq, Hq, d = q.shape
    Hkv = k_pool.shape[1]
    if max_kv_len is None:
        max_kv_len = int(kv_lens.max().item()) if kv_lens.numel() else 0
    need = attention_workspace_bytes(S, Tq, Hq, max_kv_len)
    if workspace is None:
        workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=q.device)
    _ok(_lib.load().fb_launch_attention_paged(
        q.data_ptr(), _dt(q), S, Tq, Hq, Hkv, d, k_pool.data_ptr(), v_pool.data_ptr(), k_pool.shape[0],
        block_tables.data_ptr(), block_tables.shape[1], kv_lens.data_ptr(), start_pos.data_ptr(), max_kv_len,
        workspace.data_ptr(), workspace.numel(), out.data_ptr(), _stream(stream)), "attention_paged")


# host tables -------------------------------------------------------------------

def rope_freqs(head_dim: int, theta: float) -> np.ndarray:
    out = np.zeros(head_dim // 2, dtype=np.float32)
    _ok(_lib.load().fb_rope_freqs(head_dim, theta, out.ctypes.data_as(_lib.f32p)), "fb_rope_freqs")
    return out


def rope_freqs_llama3(head_dim, theta, factor, low, high, original_max_position) -> np.ndarray:
    out = np.zeros(head_dim // 2, dtype=np.float32)
    _ok(_lib.load().fb_rope_freqs_llama3(head_dim, theta, factor, low, high, original_max_position,
                                         out.ctypes.data_as(_lib.f32p)), "fb_rope_freqs_llama3")
    return out


def gguf_rope_params(path) -> dict:
    """The rope metadata of a GGUF file (fb_gguf_rope_params)."""
    p = _lib.FbRopeParams()
    lib = _lib.load()
    if lib.fb_gguf_rope_params(str(path).encode(), C.byref(p)) != 0:
        raise ValueError(lib.fb_gguf_last_error().decode())
    d = {n: getattr(p, n) for n, _ in p._fields_ if n != "pad0"}
    d["scaling"] = _lib.FB_ROPE_SCALING[d["scaling"]]
    return d


def rope_freqs_from_gguf(path, head_dim: int) -> np.ndarray:
    """The RoPE frequency table a GGUF model file calls for (fb_rope_freqs_from_gguf)."""
    out = np.empty(head_dim // 2, dtype=np.float32)
    lib = _lib.load()
    if lib.fb_rope_freqs_from_gguf(str(path).encode(), head_dim, out.ctypes.data_as(_lib.f32p)) != 0:
        raise ValueError(lib.fb_gguf_last_error().decode())
    return out


def tq_codebook(dim: int, bits: int):
    c = np.zeros(1 << bits, dtype=np.float32)
    b = np.zeros((1 << bits) - 1, dtype=np.float32)
    _ok(_lib.load().fb_tq_codebook(dim, bits, c.ctypes.data_as(_lib.f32p), b.ctypes.data_as(_lib.f32p)),
        "fb_tq_codebook")
    return c, b


def tq_rotation_matrix(d: int, seed: int) -> np.ndarray:
    out = np.zeros((d, d), dtype=np.float32)
    _ok(_lib.load().fb_tq_rotation_matrix(d, seed, out.ctypes.data_as(_lib.f32p)), "fb_tq_rotation_matrix")
    return out
