"""Restatement of the reference's TurboQuant math and its paged quantized cache.

Test infrastructure only (see ``oracle/__init__.py``).

Follows, line by line in meaning (paths relative to the Fracture repository):

* ``TurboQuantConfig`` and helpers — ``crates/fracture-core/src/turboquant.rs:7-151``
* ``LloydMaxCodebook::compute`` (Simpson's rule, 500 points, tol 1e-10,
  200 iterations) — ``turboquant.rs:162-256``
* ``generate_rotation_matrix`` (Xoshiro256** seeded by SplitMix64, Box-Muller,
  modified Gram-Schmidt in f64, positive-diagonal sign fix) — ``turboquant.rs:306-438``
* ``rotation_seeds`` — ``turboquant.rs:341-345``
* compress arithmetic — the reference's CPU statement of the kernel in its
  tests, ``turboquant.rs:1225-1290`` (4-bit) and ``:1056-1100`` (2-bit): float32
  norm from a sequential sum of squares, ``x / (norm + 1e-8)`` by true division,
  ``y_i = sum_j Pi[i,j] * x_j`` as a sequential float32 sum with separate
  multiply and add roundings (Rust does not contract to FMA), nearest centroid
  with the first minimum winning (``turboquant_compress.cu:113-186`` uses strict
  ``<``).
* bit packing — MSB-first: 4-bit high nibble = even coordinate
  (``turboquant_compress.cu:145-146``), 2-bit shift ``6 - 2*sub`` (``:167``),
  8-bit one byte (``:175-185``). The 3-bit width has no reference layout; this
  build defines it as the same MSB-first continuous bit stream, which the 2-,
  4- and 8-bit layouts are special cases of.
* decompress — ``turboquant_decompress.cu:40-93``.
* paged write — ``crates/fracture-engine/src/quantized_paged_kv_cache.rs:404-500``
  with ``BLOCK_SIZE = 16`` (``paged_kv_cache.rs:7``).

The sequential float32 sums are written with ``np.add.accumulate``-free
explicit loops over the reduction index, vectorised over the other axes, so
each partial sum is rounded to float32 in the same order as the Rust loops.
"""

from __future__ import annotations

import ctypes
import math
import os
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

BLOCK_SIZE = 16
TQ_EPSILON = np.float32(1e-8)
MASK64 = (1 << 64) - 1

# ── config ───────────────────────────────────────────────────────────────────

REFERENCE_VALID_BITS = (2, 4, 8)
# The build also supports 3 bits; the reference rejects it.
BUILD_VALID_BITS = (2, 3, 4, 8)


class ConfigError(ValueError):
    pass


@dataclass
class TurboQuantConfig:
    key_bits: int = 4
    value_bits: int = 2
    protected_bits: int = 8
    protected_layers: int = 0
    residual_tokens: int = 0
    seed: int = 42

    def validate(self, allowed=REFERENCE_VALID_BITS) -> None:
        for name in ("key_bits", "value_bits", "protected_bits"):
            v = getattr(self, name)
            if v not in allowed:
                raise ConfigError(f"TurboQuant {name} must be one of {allowed}, got {v}")

    def is_protected(self, layer: int, num_layers: int) -> bool:
        return self.protected_layers > 0 and (
            layer < self.protected_layers or layer >= max(num_layers - self.protected_layers, 0))

    def key_bits_for_layer(self, layer: int, num_layers: int) -> int:
        return self.protected_bits if self.is_protected(layer, num_layers) else self.key_bits

    def value_bits_for_layer(self, layer: int, num_layers: int) -> int:
        return self.protected_bits if self.is_protected(layer, num_layers) else self.value_bits

    def distinct_bit_widths(self) -> list[int]:
        bits = [self.key_bits, self.value_bits]
        if self.protected_layers > 0:
            bits.append(self.protected_bits)
        return sorted(set(bits))

    @staticmethod
    def packed_dim_per_head(head_dim: int, bits: int) -> int:
        return (head_dim * bits + 7) // 8

    @staticmethod
    def bytes_per_block_layer(num_kv_heads: int, head_dim: int, key_bits: int, value_bits: int) -> int:
        kp = BLOCK_SIZE * num_kv_heads * TurboQuantConfig.packed_dim_per_head(head_dim, key_bits)
        vp = BLOCK_SIZE * num_kv_heads * TurboQuantConfig.packed_dim_per_head(head_dim, value_bits)
        return kp + vp + 2 * BLOCK_SIZE * num_kv_heads * 2

    def bytes_per_block_total(self, num_layers: int, num_kv_heads: int, head_dim: int) -> int:
        return sum(self.bytes_per_block_layer(num_kv_heads, head_dim,
                                              self.key_bits_for_layer(l, num_layers),
                                              self.value_bits_for_layer(l, num_layers))
                   for l in range(num_layers))

    def compute_num_blocks(self, gpu_available: int, scratch_reserve: int, num_layers: int,
                           num_kv_heads: int, head_dim: int) -> int:
        budget = max(gpu_available - scratch_reserve, 0)
        per = self.bytes_per_block_total(num_layers, num_kv_heads, head_dim)
        return 0 if per == 0 else budget // per


# ── Lloyd-Max codebook ───────────────────────────────────────────────────────

def _gaussian_pdf(x: float, sigma2: float) -> float:
    return (1.0 / math.sqrt(2.0 * math.pi * sigma2)) * math.exp(-x * x / (2.0 * sigma2))


def _integrate_simpson(f, a: float, b: float, n: int) -> float:
    n = n + 1 if n % 2 == 1 else n
    h = (b - a) / n
    s = f(a) + f(b)
    for i in range(1, n):
        x = a + i * h
        s += 2.0 * f(x) if i % 2 == 0 else 4.0 * f(x)
    return s * h / 3.0


@dataclass
class LloydMaxCodebook:
    centroids: np.ndarray  # float32 [2^bits]
    boundaries: np.ndarray  # float32 [2^bits - 1], f64 midpoints cast to f32
    bits: int
    dim: int

    @property
    def n_levels(self) -> int:
        return 1 << self.bits

    @staticmethod
    def compute(dim: int, bits: int) -> "LloydMaxCodebook":
        n = 1 << bits
        sigma2 = 1.0 / dim
        sigma = math.sqrt(sigma2)
        lo, hi = -3.5 * sigma, 3.5 * sigma
        c = [lo + (hi - lo) * (i + 0.5) / n for i in range(n)]
        for _ in range(200):
            b = [(c[i] + c[i + 1]) / 2.0 for i in range(n - 1)]
            elo, ehi = lo * 3.0, hi * 3.0
            new = []
            max_shift = 0.0
            for i in range(n):
                a_ = elo if i == 0 else b[i - 1]
                b_ = ehi if i == n - 1 else b[i]
                num = _integrate_simpson(lambda x: x * _gaussian_pdf(x, sigma2), a_, b_, 500)
                den = _integrate_simpson(lambda x: _gaussian_pdf(x, sigma2), a_, b_, 500)
                nc = num / den if abs(den) > 1e-15 else c[i]
                max_shift = max(max_shift, abs(nc - c[i]))
                new.append(nc)
            c = new
            if max_shift < 1e-10:
                break
        b = [(c[i] + c[i + 1]) / 2.0 for i in range(n - 1)]
        return LloydMaxCodebook(np.array(c, dtype=np.float32), np.array(b, dtype=np.float32), bits, dim)


_CODEBOOK_CACHE: dict[tuple[int, int], LloydMaxCodebook] = {}


def get_codebook(dim: int, bits: int) -> LloydMaxCodebook:
    """``get_codebook`` (turboquant.rs:278-286): the solver output for any (dim, bits)."""
    key = (dim, bits)
    if key not in _CODEBOOK_CACHE:
        _CODEBOOK_CACHE[key] = LloydMaxCodebook.compute(dim, bits)
    return _CODEBOOK_CACHE[key]


# ── Haar rotation ────────────────────────────────────────────────────────────

class Xoshiro256:
    """Xoshiro256** seeded through SplitMix64 (turboquant.rs:349-385)."""

    def __init__(self, seed: int):
        sm = seed & MASK64
        s = []
        for _ in range(4):
            sm = (sm + 0x9E3779B97F4A7C15) & MASK64
            z = sm
            z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
            z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
            z ^= z >> 31
            s.append(z)
        self.s = s

    @staticmethod
    def _rotl(x: int, k: int) -> int:
        return ((x << k) | (x >> (64 - k))) & MASK64

    def next_u64(self) -> int:
        s = self.s
        result = (self._rotl((s[1] * 5) & MASK64, 7) * 9) & MASK64
        t = (s[1] << 17) & MASK64
        s[2] ^= s[0]
        s[3] ^= s[1]
        s[1] ^= s[2]
        s[0] ^= s[3]
        s[2] ^= t
        s[3] = self._rotl(s[3], 45)
        return result

    def next_f64(self) -> float:
        return float(self.next_u64() >> 11) / float(1 << 53)


def box_muller(rng: Xoshiro256) -> tuple[np.float32, np.float32]:
    u1 = max(rng.next_f64(), 1e-15)
    u2 = rng.next_f64()
    r = math.sqrt(-2.0 * math.log(u1))
    th = 2.0 * math.pi * u2
    return np.float32(r * math.cos(th)), np.float32(r * math.sin(th))


def _seq_sum_f64_cols(m: np.ndarray) -> np.ndarray:
    """Sequential (row 0, 1, ...) f64 sum down each column of ``m``."""
    acc = np.zeros(m.shape[1:], dtype=np.float64)
    for r in range(m.shape[0]):
        acc = acc + m[r]
    return acc


def qr_orthogonalize(g: np.ndarray, d: int) -> np.ndarray:
    """Modified Gram-Schmidt in f64 (turboquant.rs:399-438); returns row-major f32 [d, d]."""
    cols = np.asarray(g, dtype=np.float32).reshape(d, d).T.astype(np.float64).copy()  # cols[col][row]
    for i in range(d):
        norm = math.sqrt(float(_seq_sum_f64_cols((cols[i] * cols[i])[:, None])[0]))
        if norm > 1e-12:
            cols[i] = cols[i] / norm
        if i + 1 < d:
            prods = cols[i + 1:] * cols[i][None, :]  # [j, row]
            dots = _seq_sum_f64_cols(prods.T)  # sequential over rows, per j
            cols[i + 1:] = cols[i + 1:] - dots[:, None] * cols[i][None, :]
    return cols.T.astype(np.float32).copy()


def generate_rotation_matrix(d: int, seed: int) -> np.ndarray:
    """Row-major float32 ``[d, d]`` Haar rotation (turboquant.rs:306-338)."""
    rng = Xoshiro256(seed)
    n = d * d
    g: list[np.float32] = []
    for _ in range((n + 1) // 2):
        z0, z1 = box_muller(rng)
        g.append(z0)
        if len(g) < n:
            g.append(z1)
    q = qr_orthogonalize(np.array(g, dtype=np.float32), d)
    for col in range(d):
        if q[col, col] < 0.0:
            q[:, col] = -q[:, col]
    return q


def rotation_seeds(base_seed: int, layer: int) -> tuple[int, int]:
    return base_seed + layer * 1000, base_seed + layer * 1000 + 500


# ── compress / decompress arithmetic ─────────────────────────────────────────

def seq_sum_f32(terms: np.ndarray) -> np.ndarray:
    """Sequential float32 sum over the LAST axis, one rounding per addition."""
    acc = np.zeros(terms.shape[:-1], dtype=np.float32)
    for j in range(terms.shape[-1]):
        acc = (acc + terms[..., j]).astype(np.float32)
    return acc


def tq_norms(x: np.ndarray) -> np.ndarray:
    """float32 L2 norm of each vector (last axis), sequential non-fused sum of squares."""
    x = np.asarray(x, dtype=np.float32)
    return np.sqrt(seq_sum_f32((x * x).astype(np.float32))).astype(np.float32)


def tq_rotate(x: np.ndarray, rotation: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Return ``(norm, y)`` for vectors ``x [..., d]``: ``y = Pi @ (x / (norm + 1e-8))``."""
    x = np.asarray(x, dtype=np.float32)
    d = x.shape[-1]
    norm = tq_norms(x)
    xn = (x / (norm[..., None] + TQ_EPSILON).astype(np.float32)).astype(np.float32)
    pi = np.asarray(rotation, dtype=np.float32).reshape(d, d)
    acc = np.zeros(x.shape[:-1] + (d,), dtype=np.float32)
    for j in range(d):
        acc = (acc + (pi[None, :, j] * xn[..., j, None]).astype(np.float32)).astype(np.float32)
    return norm, acc


def nearest_centroid(y: np.ndarray, centroids: np.ndarray) -> np.ndarray:
    """Index of the nearest centroid with the first minimum winning (strict ``<``)."""
    c = np.asarray(centroids, dtype=np.float32)
    y = np.asarray(y, dtype=np.float32)
    best = np.abs((y - c[0]).astype(np.float32))
    idx = np.zeros(y.shape, dtype=np.int32)
    for k in range(1, c.shape[0]):
        dist = np.abs((y - c[k]).astype(np.float32))
        better = dist < best
        best = np.where(better, dist, best)
        idx = np.where(better, k, idx)
    return idx


def pack_indices(idx: np.ndarray, bits: int) -> np.ndarray:
    """MSB-first bit stream per vector (last axis) -> uint8 ``[..., ceil(d*bits/8)]``."""
    idx = np.asarray(idx, dtype=np.uint32)
    d = idx.shape[-1]
    nbytes = (d * bits + 7) // 8
    bitplanes = ((idx[..., :, None] >> np.arange(bits - 1, -1, -1, dtype=np.uint32)) & 1).astype(np.uint8)
    stream = bitplanes.reshape(idx.shape[:-1] + (d * bits,))
    pad = nbytes * 8 - d * bits
    if pad:
        stream = np.concatenate([stream, np.zeros(idx.shape[:-1] + (pad,), np.uint8)], axis=-1)
    return np.packbits(stream, axis=-1, bitorder="big")


def unpack_indices(packed: np.ndarray, bits: int, d: int) -> np.ndarray:
    packed = np.asarray(packed, dtype=np.uint8)
    stream = np.unpackbits(packed, axis=-1, bitorder="big")[..., : d * bits]
    planes = stream.reshape(packed.shape[:-1] + (d, bits)).astype(np.uint32)
    weights = (1 << np.arange(bits - 1, -1, -1, dtype=np.uint32))
    return (planes * weights).sum(axis=-1).astype(np.int32)


def compress(x: np.ndarray, rotation: np.ndarray, centroids: np.ndarray, bits: int):
    """TurboQuant compress of ``x [N, H, d]`` (values of the fp16/bf16 input).

    Returns ``(packed uint8 [N, H*P], norms float32 [N, H] (values), idx int32 [N, H, d], y float32)``
    where the norms are rounded to float16 as the reference stores them.
    """
    x = np.asarray(x, dtype=np.float32)
    N, H, d = x.shape
    norm, y = tq_rotate(x, rotation)
    idx = nearest_centroid(y, centroids)
    packed = pack_indices(idx, bits).reshape(N, H * TurboQuantConfig.packed_dim_per_head(d, bits))
    norms16 = norm.astype(np.float16).astype(np.float32)
    return packed, norms16, idx, y


def decompress(packed: np.ndarray, norms: np.ndarray, rotation: np.ndarray, centroids: np.ndarray,
               bits: int, num_kv_heads: int, head_dim: int) -> np.ndarray:
    """``x_hat = Pi^T @ centroids[idx]`` times the stored norm, float32 sequential sums."""
    d = head_dim
    P = TurboQuantConfig.packed_dim_per_head(d, bits)
    packed = np.asarray(packed, dtype=np.uint8).reshape(-1, num_kv_heads, P)
    idx = unpack_indices(packed, bits, d)
    yh = np.asarray(centroids, dtype=np.float32)[idx]
    pi = np.asarray(rotation, dtype=np.float32).reshape(d, d)
    acc = np.zeros(yh.shape, dtype=np.float32)
    for j in range(d):
        acc = (acc + (pi[None, None, j, :] * yh[..., j, None]).astype(np.float32)).astype(np.float32)
    nrm = np.asarray(norms, dtype=np.float32).reshape(acc.shape[:-1])
    return (acc * nrm[..., None]).astype(np.float32)


# ── decision-boundary distance (for tie accounting) ─────────────────────────

def boundary_distance(y: np.ndarray, centroids: np.ndarray) -> np.ndarray:
    """Distance of each coordinate to the nearest midpoint between adjacent centroids."""
    c = np.asarray(centroids, dtype=np.float64)
    mids = (c[:-1] + c[1:]) / 2.0
    yy = np.asarray(y, dtype=np.float64)[..., None]
    return np.min(np.abs(yy - mids), axis=-1)


# ── C version of the exact compress (fast, for larger parity checks) ────────

_LIB = None


def c_oracle():
    """ctypes handle to ``oracle/_build/libtq_oracle.so`` (built by ``oracle/Makefile``)."""
    global _LIB
    if _LIB is None:
        path = Path(__file__).resolve().parent / "_build" / "libtq_oracle.so"
        if not path.exists():
            raise FileNotFoundError(f"{path} missing: run `make -C oracle`")
        lib = ctypes.CDLL(str(path))
        lib.tq_oracle_compress.restype = ctypes.c_int
        lib.tq_oracle_compress.argtypes = [
            ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_long, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        lib.tq_oracle_decompress.restype = ctypes.c_int
        lib.tq_oracle_decompress.argtypes = [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_long, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        _LIB = lib
    return _LIB


INPUT_F16, INPUT_BF16, INPUT_F32 = 0, 1, 2


def compress_c(x_bits: np.ndarray, input_kind: int, rotation: np.ndarray, centroids: np.ndarray,
               bits: int, num_threads: int = 1):
    """Exact compress in C. ``x_bits``: uint16 raw fp16/bf16 bits (or float32) ``[N, H, d]``.

    Returns ``(packed uint8 [N, H*P], norm_f16_bits uint16 [N, H], idx uint8 [N, H, d])``.
    """
    lib = c_oracle()
    x_bits = np.ascontiguousarray(x_bits)
    N, H, d = x_bits.shape
    P = TurboQuantConfig.packed_dim_per_head(d, bits)
    rot = np.ascontiguousarray(rotation, dtype=np.float32)
    cen = np.ascontiguousarray(centroids, dtype=np.float32)
    packed = np.zeros((N, H * P), dtype=np.uint8)
    norms = np.zeros((N, H), dtype=np.uint16)
    idx = np.zeros((N, H, d), dtype=np.uint8)
    rc = lib.tq_oracle_compress(x_bits.ctypes.data, input_kind, rot.ctypes.data, cen.ctypes.data,
                                cen.shape[0], packed.ctypes.data, norms.ctypes.data, idx.ctypes.data,
                                N, H, d, bits, num_threads)
    if rc != 0:
        raise RuntimeError(f"tq_oracle_compress failed: {rc}")
    return packed, norms, idx


def decompress_c(packed: np.ndarray, norm_f16_bits: np.ndarray, rotation: np.ndarray,
                 centroids: np.ndarray, bits: int, num_kv_heads: int, head_dim: int,
                 num_threads: int = 1) -> np.ndarray:
    lib = c_oracle()
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    norms = np.ascontiguousarray(norm_f16_bits, dtype=np.uint16)
    N = packed.shape[0]
    rot = np.ascontiguousarray(rotation, dtype=np.float32)
    cen = np.ascontiguousarray(centroids, dtype=np.float32)
    out = np.zeros((N, num_kv_heads, head_dim), dtype=np.float32)
    rc = lib.tq_oracle_decompress(packed.ctypes.data, norms.ctypes.data, rot.ctypes.data,
                                  cen.ctypes.data, out.ctypes.data, N, num_kv_heads, head_dim, bits,
                                  num_threads)
    if rc != 0:
        raise RuntimeError(f"tq_oracle_decompress failed: {rc}")
    return out


# ── paged quantized cache (block accounting + placement) ────────────────────

@dataclass
class _Seq:
    block_table: list[int]
    last_block_fill: int = 0
    current_len: int = 0


@dataclass
class QuantizedKvCache:
    """Block accounting of ``QuantizedKvCacheManager`` plus a host copy of the pool.

    ``pool_packed[layer][kv]`` is ``[num_blocks*16, H*P]`` uint8 and
    ``pool_norms[layer][kv]`` is ``[num_blocks*16, H]`` uint16 (fp16 bits):
    block ``b`` occupies rows ``16*b .. 16*b+15``, the same per-block layout as the
    reference's ``[BLOCK_SIZE, num_kv_heads * packed_dim]`` INT8 block tensors
    (``quantized_paged_kv_cache.rs:82-133``) placed back to back.
    """

    num_blocks: int
    num_layers: int
    num_kv_heads: int
    head_dim: int
    config: TurboQuantConfig
    free_list: list[int] = field(default_factory=list)
    seqs: dict[int, _Seq] = field(default_factory=dict)
    next_id: int = 0

    def __post_init__(self):
        self.free_list = list(range(self.num_blocks))[::-1]
        self.key_bits = [self.config.key_bits_for_layer(l, self.num_layers) for l in range(self.num_layers)]
        self.value_bits = [self.config.value_bits_for_layer(l, self.num_layers) for l in range(self.num_layers)]
        rows = self.num_blocks * BLOCK_SIZE
        self.pool_packed = []
        self.pool_norms = []
        for l in range(self.num_layers):
            kb, vb = self.key_bits[l], self.value_bits[l]
            self.pool_packed.append([
                np.zeros((rows, self.num_kv_heads * TurboQuantConfig.packed_dim_per_head(self.head_dim, kb)), np.uint8),
                np.zeros((rows, self.num_kv_heads * TurboQuantConfig.packed_dim_per_head(self.head_dim, vb)), np.uint8)])
            self.pool_norms.append([np.zeros((rows, self.num_kv_heads), np.uint16),
                                    np.zeros((rows, self.num_kv_heads), np.uint16)])

    def _alloc_block(self) -> int:
        if not self.free_list:
            raise MemoryError("out of quantized KV blocks")
        return self.free_list.pop()

    def alloc(self) -> int:
        sid = self.next_id
        self.next_id += 1
        self.seqs[sid] = _Seq(block_table=[self._alloc_block()])
        return sid

    def free(self, sid: int) -> None:
        seq = self.seqs.pop(sid)
        for b in seq.block_table:
            self.free_list.append(b)

    def reserve(self, sid: int, num_new: int) -> int:
        """Layer-0 block growth of ``append_kv`` (rs:446-465); returns the start position."""
        seq = self.seqs[sid]
        remaining, fill = num_new, seq.last_block_fill
        while remaining > 0:
            slots = BLOCK_SIZE - fill
            if slots == 0:
                seq.block_table.append(self._alloc_block())
                fill = 0
                continue
            w = min(remaining, slots)
            fill += w
            remaining -= w
        seq.last_block_fill = fill
        seq.current_len += num_new
        return seq.current_len - num_new

    def slots(self, sid: int, start: int, num_new: int) -> np.ndarray:
        """Physical pool row of each new token (rs:471-497)."""
        bt = self.seqs[sid].block_table
        pos = start + np.arange(num_new)
        return np.array([bt[p // BLOCK_SIZE] * BLOCK_SIZE + p % BLOCK_SIZE for p in pos], dtype=np.int64)

    def append_kv(self, sid: int, layer: int, k_packed, k_norms, v_packed, v_norms) -> None:
        """Place already-compressed rows (the reference's scratch tensors) into the pool."""
        n = k_packed.shape[0]
        if layer == 0:
            self.reserve(sid, n)
        start = self.seqs[sid].current_len - n
        rows = self.slots(sid, start, n)
        self.pool_packed[layer][0][rows] = k_packed
        self.pool_norms[layer][0][rows] = k_norms
        self.pool_packed[layer][1][rows] = v_packed
        self.pool_norms[layer][1][rows] = v_norms


# ── paged attention over the compressed cache ───────────────────────────────

def attention_paged_tq(q: np.ndarray, k_packed: np.ndarray, k_norms: np.ndarray, v_packed: np.ndarray,
                       v_norms: np.ndarray, block_table: np.ndarray, kv_len: int, start_pos: int,
                       k_rotation: np.ndarray, v_rotation: np.ndarray, k_centroids: np.ndarray,
                       v_centroids: np.ndarray, key_bits: int, value_bits: int, num_kv_heads: int) -> np.ndarray:
    """The statement of ``attention_paged_tq_kernel`` (``backends/fracture-cuda/kernels/
    attention_paged_tq.cu:56-257``) in float64, for one sequence.

    ``q [N, Hq, d]`` (values); pools ``[rows, Hkv * P]`` uint8 with norms ``[rows, Hkv]`` (values)
    addressed by ``block_table[pos // 16] * 16 + pos % 16``. Query token t attends positions
    ``[0, min(start_pos + t + 1, kv_len))`` (``:86-87``); q head h reads KV head
    ``h // (Hq / Hkv)`` (``:83-84``). Scores in K's rotated space,
    ``(Pi_k q) . c_k[idx] * k_norm / sqrt(d)`` (``:102-140``); softmax (``:145-206``); values
    accumulated in V's rotated space, ``sum p * c_v[idx] * v_norm``, then ``Pi_v^T @ acc``
    (``:208-280``). A position whose block-table entry is negative is left out (the reference
    has no such case). A query with no position gives zeros.
    """
    q = np.asarray(q, np.float64)
    N, Hq, d = q.shape
    G = Hq // num_kv_heads
    Pk, Pv = (d * key_bits + 7) // 8, (d * value_bits + 7) // 8
    kp = np.asarray(k_packed, np.uint8).reshape(-1, num_kv_heads, Pk)
    vp = np.asarray(v_packed, np.uint8).reshape(-1, num_kv_heads, Pv)
    kn = np.asarray(k_norms, np.float64).reshape(-1, num_kv_heads)
    vn = np.asarray(v_norms, np.float64).reshape(-1, num_kv_heads)
    pik, piv = np.asarray(k_rotation, np.float64), np.asarray(v_rotation, np.float64)
    ck, cv = np.asarray(k_centroids, np.float64), np.asarray(v_centroids, np.float64)
    table = np.asarray(block_table, np.int64)
    out = np.zeros((N, Hq, d), np.float64)
    scale = 1.0 / np.sqrt(d)
    for t in range(N):
        L = min(start_pos + t + 1, kv_len)
        pos = np.arange(L)
        blk = table[pos // 16]
        keep = blk >= 0
        rows = (blk * 16 + pos % 16)[keep]
        for g in range(num_kv_heads):
            if rows.size == 0:
                continue
            yk = ck[unpack_indices(kp[rows, g], key_bits, d)]      # [L', d]
            yv = cv[unpack_indices(vp[rows, g], value_bits, d)]
            for h in range(g * G, (g + 1) * G):
                qr = pik @ q[t, h]
                s = (yk @ qr) * kn[rows, g] * scale
                p = np.exp(s - s.max())
                p /= p.sum()
                acc = (p * vn[rows, g]) @ yv
                out[t, h] = piv.T @ acc
    return out
