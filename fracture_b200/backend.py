"""Python face of the backend object: the reference's ``Backend`` trait over the C ABI.

Mirrors ``trait Backend`` (crates/fracture-core/src/backend.rs:8-223) and
``CudaBackend`` (backends/fracture-cuda/src/{lib,backend}.rs): opaque
``DeviceTensor`` handles, the same method names and argument meaning, and one
exception class per ``FractureError`` variant (crates/fracture-core/src/
error.rs:7-50). All work happens in ``libfracture_b200.so``; this module only
marshals arguments.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import FB_BF16, FB_FP16, FB_FP32, FB_INT4, FB_INT8, FbTensor, FbTqConfig


class FractureError(Exception):
    """Base class; ``str(e)`` carries the backend's message."""


class BackendError(FractureError):
    pass


class OutOfMemory(FractureError):
    pass


class InvalidShape(FractureError):
    pass


class TensorNotFound(FractureError):
    pass


class UnsupportedDType(FractureError):
    pass


class KvCacheError(FractureError):
    pass


class ModelConfigError(FractureError):
    pass


_STATUS = {1: BackendError, 2: OutOfMemory, 3: InvalidShape, 4: TensorNotFound, 5: UnsupportedDType,
           6: KvCacheError, 7: ModelConfigError}

DTYPE_SIZE = {FB_FP16: 2, FB_FP32: 4, FB_BF16: 2, FB_INT8: 1, FB_INT4: 1}
DTYPE_NAME = {FB_FP16: "fp16", FB_FP32: "fp32", FB_BF16: "bf16", FB_INT8: "int8", FB_INT4: "int4"}


def _check(rc: int) -> None:
    if rc != 0:
        msg = _lib.load().fb_last_error().decode(errors="replace")
        raise _STATUS.get(rc, FractureError)(msg)


@dataclass(frozen=True)
class DeviceTensor:
    """``DeviceTensor {id, shape, dtype}`` (crates/fracture-core/src/tensor.rs:14-18)."""

    id: int
    shape: tuple
    dtype: int

    def numel(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 0

    def size_bytes(self) -> int:
        n = self.numel()
        return (n + 1) // 2 if self.dtype == FB_INT4 else n * DTYPE_SIZE[self.dtype]

    def reshape(self, shape) -> "DeviceTensor":
        shape = tuple(int(s) for s in shape)
        if int(np.prod(shape)) != self.numel():
            raise InvalidShape(f"cannot reshape tensor with {self.numel()} elements to shape {list(shape)}")
        return DeviceTensor(self.id, shape, self.dtype)

    def c(self) -> FbTensor:
        t = FbTensor()
        t.id = self.id
        t.dtype = self.dtype
        t.ndim = len(self.shape)
        for i, s in enumerate(self.shape):
            t.shape[i] = int(s)
        return t


def _ref(t: DeviceTensor):
    return C.byref(t.c())


class CudaBackend:
    """``CudaBackend::new(device)`` with the trait methods of the hot path."""

    def __init__(self, device: int = 0):
        self._lib = _lib.load()
        h = C.c_void_p()
        _check(self._lib.fb_backend_create(device, C.byref(h)))
        self._h = h

    # lifecycle ---------------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.fb_backend_destroy(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def stream(self) -> int:
        s = C.c_void_p()
        _check(self._lib.fb_backend_stream(self._h, C.byref(s)))
        return s.value or 0

    def device_name(self) -> str:
        buf = C.create_string_buffer(256)
        _check(self._lib.fb_backend_device_name(self._h, buf, 256))
        return buf.value.decode()

    def total_memory(self) -> int:
        v = C.c_size_t()
        _check(self._lib.fb_backend_total_memory(self._h, C.byref(v)))
        return v.value

    def available_memory(self) -> int:
        v = C.c_size_t()
        _check(self._lib.fb_backend_available_memory(self._h, C.byref(v)))
        return v.value

    # memory ------------------------------------------------------------------
    def alloc(self, shape, dtype: int) -> DeviceTensor:
        shape = tuple(int(s) for s in shape)
        arr = (C.c_int64 * max(len(shape), 1))(*shape)
        out = FbTensor()
        _check(self._lib.fb_alloc(self._h, arr, len(shape), dtype, C.byref(out)))
        return DeviceTensor(out.id, shape, dtype)

    def register_external(self, ptr: int, shape, dtype: int) -> DeviceTensor:
        shape = tuple(int(s) for s in shape)
        arr = (C.c_int64 * len(shape))(*shape)
        out = FbTensor()
        _check(self._lib.fb_register_external(self._h, C.c_void_p(ptr), arr, len(shape), dtype, C.byref(out)))
        return DeviceTensor(out.id, shape, dtype)

    def get_ptr(self, t: DeviceTensor) -> int:
        p = C.c_void_p()
        _check(self._lib.fb_get_ptr(self._h, _ref(t), C.byref(p)))
        return p.value or 0

    def free(self, t: DeviceTensor) -> None:
        _check(self._lib.fb_free(self._h, _ref(t)))

    def copy_to_device(self, dst: DeviceTensor, src) -> None:
        buf = np.ascontiguousarray(src).view(np.uint8).ravel()
        _check(self._lib.fb_copy_to_device(self._h, _ref(dst), buf.ctypes.data, buf.nbytes))

    def copy_to_host(self, src: DeviceTensor, dst: np.ndarray | None = None) -> np.ndarray:
        if dst is None:
            dst = np.empty(src.size_bytes(), dtype=np.uint8)
        buf = dst.view(np.uint8).reshape(-1)
        _check(self._lib.fb_copy_to_host(self._h, _ref(src), buf.ctypes.data, buf.nbytes))
        return dst

    # compute -----------------------------------------------------------------
    def rmsnorm(self, input: DeviceTensor, weight: DeviceTensor, eps: float, out: DeviceTensor) -> None:
        _check(self._lib.fb_rmsnorm(self._h, _ref(input), _ref(weight), float(eps), _ref(out)))

    def rope(self, q: DeviceTensor, k: DeviceTensor, positions, theta: float, head_dim: int) -> None:
        pos = np.ascontiguousarray(positions, dtype=np.uint32)
        _check(self._lib.fb_rope(self._h, _ref(q), _ref(k), pos.ctypes.data_as(_lib.u32p), pos.size, float(theta),
                                 int(head_dim)))

    def silu_mul(self, gate: DeviceTensor, up: DeviceTensor, out: DeviceTensor) -> None:
        _check(self._lib.fb_silu_mul(self._h, _ref(gate), _ref(up), _ref(out)))

    def embedding(self, token_ids, embedding_table: DeviceTensor, out: DeviceTensor) -> None:
        ids = np.ascontiguousarray(token_ids, dtype=np.uint32)
        _check(self._lib.fb_embedding(self._h, ids.ctypes.data_as(_lib.u32p), ids.size, _ref(embedding_table),
                                      _ref(out)))

    def add(self, a: DeviceTensor, b: DeviceTensor, out: DeviceTensor) -> None:
        _check(self._lib.fb_add(self._h, _ref(a), _ref(b), _ref(out)))

    def copy_rows(self, src: DeviceTensor, dst: DeviceTensor, src_offset: int, dst_offset: int, count: int) -> None:
        _check(self._lib.fb_copy_rows(self._h, _ref(src), _ref(dst), src_offset, dst_offset, count))

    def turboquant_compress(self, input: DeviceTensor, rotation_matrix: DeviceTensor, centroids: DeviceTensor,
                            bits: int, packed_out: DeviceTensor, norms_out: DeviceTensor) -> None:
        _check(self._lib.fb_turboquant_compress(self._h, _ref(input), _ref(rotation_matrix), _ref(centroids), bits,
                                                _ref(packed_out), _ref(norms_out)))

    def synchronize(self) -> None:
        _check(self._lib.fb_synchronize(self._h))

    def precompute_rope_freqs(self, head_dim: int, theta: float) -> None:
        _check(self._lib.fb_precompute_rope_freqs(self._h, head_dim, float(theta)))

    def precompute_rope_freqs_llama3(self, head_dim: int, theta: float, factor: float, low_freq_factor: float,
                                     high_freq_factor: float, original_max_position: int) -> None:
        _check(self._lib.fb_precompute_rope_freqs_llama3(self._h, head_dim, float(theta), float(factor),
                                                         float(low_freq_factor), float(high_freq_factor),
                                                         float(original_max_position)))

    def precompute_rope_freqs_gguf(self, head_dim: int, gguf_path) -> None:
        """The RoPE table a GGUF model file calls for (llama3 scaling from its metadata or its
        rope_freqs tensor); replaces precompute_rope_freqs(head_dim, theta) at the server's start."""
        _check(self._lib.fb_precompute_rope_freqs_gguf(self._h, head_dim, str(gguf_path).encode()))

    # timers ------------------------------------------------------------------
    def create_timer(self) -> int:
        t = C.c_uint64()
        _check(self._lib.fb_create_timer(self._h, C.byref(t)))
        return t.value

    def start_timer(self, t: int) -> None:
        _check(self._lib.fb_start_timer(self._h, t))

    def stop_timer(self, t: int) -> float:
        ms = C.c_float()
        _check(self._lib.fb_stop_timer(self._h, t, C.byref(ms)))
        return ms.value

    def destroy_timer(self, t: int) -> None:
        _check(self._lib.fb_destroy_timer(self._h, t))


class PagedKvCache:
    """``PagedKvCacheManager`` (paged_kv_cache.rs:207-370) for the uncompressed FP16/BF16 cache."""

    def __init__(self, backend: CudaBackend, num_blocks: int, num_layers: int, num_kv_heads: int, head_dim: int,
                 dtype: int = FB_FP16):
        self._lib = backend._lib
        self.backend = backend
        self.num_blocks, self.num_layers, self.num_kv_heads, self.head_dim = num_blocks, num_layers, num_kv_heads, head_dim
        h = C.c_void_p()
        _check(self._lib.fb_kv_cache_create(backend.handle, num_blocks, num_layers, num_kv_heads, head_dim, dtype,
                                            C.byref(h)))
        self._h = h

    def destroy(self) -> None:
        if self._h:
            self._lib.fb_kv_cache_destroy(self._h)
            self._h = None

    def alloc(self) -> int:
        v = C.c_uint64()
        _check(self._lib.fb_kv_cache_alloc(self._h, C.byref(v)))
        return v.value

    def free(self, handle: int) -> None:
        _check(self._lib.fb_kv_cache_free(self._h, handle))

    def append_kv(self, handle: int, layer: int, keys: DeviceTensor, values: DeviceTensor) -> None:
        _check(self._lib.fb_kv_cache_append_kv(self._h, handle, layer, _ref(keys), _ref(values)))

    def block_table(self, handle: int) -> list[int]:
        n = C.c_size_t()
        _check(self._lib.fb_kv_cache_block_table(self._h, handle, None, 0, C.byref(n)))
        arr = (C.c_int32 * max(n.value, 1))()
        _check(self._lib.fb_kv_cache_block_table(self._h, handle, arr, n.value, C.byref(n)))
        return list(arr[: n.value])

    def seq_len(self, handle: int) -> int:
        v, f = C.c_size_t(), C.c_size_t()
        _check(self._lib.fb_kv_cache_seq_len(self._h, handle, C.byref(v), C.byref(f)))
        return v.value

    def last_block_tokens(self, handle: int) -> int:
        v, f = C.c_size_t(), C.c_size_t()
        _check(self._lib.fb_kv_cache_seq_len(self._h, handle, C.byref(v), C.byref(f)))
        return f.value

    def num_free_blocks(self) -> int:
        v = C.c_size_t()
        _check(self._lib.fb_kv_cache_num_free_blocks(self._h, C.byref(v)))
        return v.value

    def pool(self, layer: int) -> dict:
        k, v = C.c_void_p(), C.c_void_p()
        _check(self._lib.fb_kv_cache_pool(self._h, layer, C.byref(k), C.byref(v)))
        return {"k": k.value, "v": v.value}

    def attention(self, handle: int, layer: int, q: DeviceTensor, kv_len: int, start_pos: int,
                  out: DeviceTensor) -> None:
        _check(self._lib.fb_kv_cache_attention(self._h, handle, layer, _ref(q), kv_len, start_pos, _ref(out)))


@dataclass
class TurboQuantConfig:
    """``TurboQuantConfig`` (crates/fracture-core/src/turboquant.rs:7-33); 3 bits is accepted here."""

    key_bits: int = 4
    value_bits: int = 2
    protected_bits: int = 8
    protected_layers: int = 0
    residual_tokens: int = 0
    seed: int = 42

    def c(self) -> FbTqConfig:
        c = FbTqConfig()
        c.key_bits, c.value_bits, c.protected_bits = self.key_bits, self.value_bits, self.protected_bits
        c.protected_layers, c.residual_tokens, c.seed = self.protected_layers, self.residual_tokens, self.seed
        return c


class QuantizedKvCache:
    """``QuantizedKvCacheManager`` with the append fused into one launch per K / V."""

    def __init__(self, backend: CudaBackend, num_blocks: int, num_layers: int, num_kv_heads: int, head_dim: int,
                 config: TurboQuantConfig | None = None):
        self._lib = backend._lib
        self.backend = backend
        self.num_blocks, self.num_layers, self.num_kv_heads, self.head_dim = num_blocks, num_layers, num_kv_heads, head_dim
        cfg = (config or TurboQuantConfig()).c()
        h = C.c_void_p()
        _check(self._lib.fb_tq_cache_create(backend.handle, num_blocks, num_layers, num_kv_heads, head_dim,
                                            C.byref(cfg), C.byref(h)))
        self._h = h

    def destroy(self) -> None:
        if self._h:
            self._lib.fb_tq_cache_destroy(self._h)
            self._h = None

    def alloc(self) -> int:
        v = C.c_uint64()
        _check(self._lib.fb_tq_cache_alloc(self._h, C.byref(v)))
        return v.value

    def free(self, handle: int) -> None:
        _check(self._lib.fb_tq_cache_free(self._h, handle))

    def append_kv(self, handle: int, layer: int, keys: DeviceTensor, values: DeviceTensor) -> None:
        _check(self._lib.fb_tq_cache_append_kv(self._h, handle, layer, _ref(keys), _ref(values)))

    def block_table(self, handle: int) -> list[int]:
        n = C.c_size_t()
        _check(self._lib.fb_tq_cache_block_table(self._h, handle, None, 0, C.byref(n)))
        arr = (C.c_int32 * max(n.value, 1))()
        _check(self._lib.fb_tq_cache_block_table(self._h, handle, arr, n.value, C.byref(n)))
        return list(arr[: n.value])

    def seq_len(self, handle: int) -> int:
        v = C.c_size_t()
        _check(self._lib.fb_tq_cache_seq_len(self._h, handle, C.byref(v)))
        return v.value

    def num_free_blocks(self) -> int:
        v = C.c_size_t()
        _check(self._lib.fb_tq_cache_num_free_blocks(self._h, C.byref(v)))
        return v.value

    def pool(self, layer: int, kv: int) -> dict:
        p, n, r, c = C.c_void_p(), C.c_void_p(), C.c_void_p(), C.c_void_p()
        bits = C.c_int()
        _check(self._lib.fb_tq_cache_pool(self._h, layer, kv, C.byref(p), C.byref(n), C.byref(r), C.byref(c),
                                          C.byref(bits)))
        return {"packed": p.value, "norms": n.value, "rotation": r.value, "centroids": c.value, "bits": bits.value}

    def dequant(self, handle: int, layer: int, kv: int, count: int, out: DeviceTensor) -> None:
        _check(self._lib.fb_tq_cache_dequant(self._h, handle, layer, kv, count, _ref(out)))

    def attention(self, handle: int, layer: int, q: DeviceTensor, kv_len: int, start_pos: int,
                  out: DeviceTensor) -> None:
        """``attention_paged_tq`` of the sequence's cached layer (``batched.rs:143-193``)."""
        _check(self._lib.fb_tq_cache_attention(self._h, handle, layer, _ref(q), kv_len, start_pos, _ref(out)))
