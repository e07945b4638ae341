"""numpy restatement of the reference's per-layer elementwise kernels.

Test infrastructure only (see ``oracle/__init__.py``). Every function works on
float32 numpy arrays that hold the *values* of the storage dtype ("f16",
"bf16" or "f32"); ``round_to`` rounds a float32 result to the storage dtype
(round-to-nearest-even) and returns it as float32 again.

Reference call sites (paths relative to the Fracture repository root):

* embedding   ``backends/fracture-cuda/kernels/embedding.cu:15-27``
* add         ``backends/fracture-cuda/kernels/add.cu:11-13`` (one rounding)
* rmsnorm     ``backends/fracture-cuda/kernels/rmsnorm.cu:24-66``
* rope        ``backends/fracture-cuda/kernels/rope.cu:38-48`` with the
              frequency table of ``backends/fracture-cuda/src/lib.rs:133-138``
* silu_mul    ``backends/fracture-cuda/kernels/silu_mul.cu:17-22``
* llama3 rope frequency rule: not in the reference (it has no RoPE scaling);
  the published Llama 3.1 rule, checked against ``transformers`` at test time.
"""

from __future__ import annotations

import math

import numpy as np

DTYPES = ("f16", "bf16", "f32")


# ── storage rounding ─────────────────────────────────────────────────────────

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 values to bfloat16 (nearest-even) and return the uint16 bits."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    r = np.where(nan, 0x7FC0, r)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to the storage dtype; return them as float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f32":
        return x.copy()
    if dtype == "f16":
        with np.errstate(over="ignore"):
            return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(x))
    raise ValueError(f"unknown dtype {dtype}")


def to_storage_bytes(x: np.ndarray, dtype: str) -> np.ndarray:
    """Encode float32 values (already representable) into the storage dtype as raw bits."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f32":
        return x.view(np.uint32)
    if dtype == "f16":
        return x.astype(np.float16).view(np.uint16)
    if dtype == "bf16":
        return f32_to_bf16_bits(x)
    raise ValueError(dtype)


# ── embedding / add ──────────────────────────────────────────────────────────

def embedding(table: np.ndarray, token_ids: np.ndarray) -> np.ndarray:
    """``out[t, :] = table[ids[t], :]``; ids >= vocab give a zero row (embedding.cu:21-25)."""
    ids = np.asarray(token_ids, dtype=np.uint64)
    vocab = table.shape[0]
    out = np.zeros((ids.shape[0], table.shape[1]), dtype=table.dtype)
    ok = ids < vocab
    out[ok] = table[ids[ok].astype(np.int64)]
    return out


def add(a: np.ndarray, b: np.ndarray, dtype: str) -> np.ndarray:
    """``out = a + b`` with one rounding to the storage dtype (add.cu:13, ``__hadd``).

    For f16/bf16 inputs the float32 sum is exact or cannot sit on a rounding
    midpoint, so rounding the float32 sum equals rounding the exact sum.
    """
    return round_to(np.asarray(a, np.float32) + np.asarray(b, np.float32), dtype)


# ── rmsnorm ──────────────────────────────────────────────────────────────────

def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float, dtype: str) -> np.ndarray:
    """``out = x * rsqrt(mean(x^2) + eps) * w`` (rmsnorm.cu:24-66).

    The sum of squares is accumulated in float64 (the FP32-or-better reference
    the tolerances are stated against); the product is rounded once to the
    storage dtype, as the kernel does (``__float2half(val * rms_inv * w)``).
    """
    x64 = np.asarray(x, np.float64)
    ms = np.mean(x64 * x64, axis=-1, keepdims=True)
    r = 1.0 / np.sqrt(ms + float(np.float32(eps)))
    out = x64 * r * np.asarray(w, np.float64)
    return round_to(out.astype(np.float32), dtype)


def add_rmsnorm(h: np.ndarray, residual: np.ndarray, w: np.ndarray, eps: float, dtype: str):
    """Fused residual add + RMSNorm, the pair ``add(h, r, h); rmsnorm(h, w, eps, out)``.

    The engine calls the two ops back to back (``crates/fracture-engine/src/
    batched.rs:393-396``, ``engine.rs:364-371``); the norm reads the *rounded*
    sum that ``add`` stored. Returns ``(h_new, normed)``.
    """
    h_new = add(h, residual, dtype)
    return h_new, rmsnorm(h_new, w, eps, dtype)


# ── rope ─────────────────────────────────────────────────────────────────────

def rope_freqs(head_dim: int, theta: float) -> np.ndarray:
    """``CudaBackend::precompute_rope_freqs`` (src/lib.rs:133-138).

    ``*freq = 1.0 / theta.powf(2.0 * i as f64 / head_dim as f64) as f32`` — the
    power is taken in f64 and cast to f32 *before* the f32 reciprocal, because
    ``as`` binds tighter than ``/`` in Rust.
    """
    half = head_dim // 2
    out = np.empty(half, dtype=np.float32)
    for i in range(half):
        p = np.float32(math.pow(theta, 2.0 * float(i) / float(head_dim)))
        out[i] = np.float32(1.0) / p
    return out


def rope_freqs_llama3(head_dim: int, theta: float, factor: float, low_freq_factor: float,
                      high_freq_factor: float, original_max_position: int) -> np.ndarray:
    """Llama 3.1 frequency scaling applied to :func:`rope_freqs`.

    Published rule (Llama 3.1 release): with ``wavelen = 2*pi/f``,
    ``f/factor`` where ``wavelen > orig/low``; ``f`` where
    ``wavelen < orig/high``; otherwise the smooth blend
    ``(1-s)*f/factor + s*f`` with ``s = (orig/wavelen - low)/(high - low)``.
    Evaluated in float64 on the float32 base frequencies, rounded to float32.
    """
    base = rope_freqs(head_dim, theta).astype(np.float64)
    low_wavelen = original_max_position / low_freq_factor
    high_wavelen = original_max_position / high_freq_factor
    out = np.empty_like(base)
    for i, f in enumerate(base):
        wavelen = 2.0 * math.pi / f
        if wavelen < high_wavelen:
            out[i] = f
        elif wavelen > low_wavelen:
            out[i] = f / factor
        else:
            s = (original_max_position / wavelen - low_freq_factor) / (high_freq_factor - low_freq_factor)
            out[i] = (1.0 - s) * f / factor + s * f
    return out.astype(np.float32)


def rope(x: np.ndarray, positions: np.ndarray, freqs: np.ndarray, dtype: str) -> np.ndarray:
    """Split-half rotary embedding (rope.cu:38-48); ``x`` is ``[T, H, d]``.

    ``angle = float(pos) * freq[d]`` is an f32 product, as in the kernel and in
    ``scripts/dump_reference.py:274-286``; cos/sin of that f32 angle are taken
    in float64 and the rotation is done in float64, rounded once.
    """
    x = np.asarray(x, np.float32)
    T, H, d = x.shape
    half = d // 2
    pos = np.asarray(positions, dtype=np.uint32).astype(np.float32)
    ang = (pos[:, None] * np.asarray(freqs, np.float32)[None, :]).astype(np.float32)
    c = np.cos(ang.astype(np.float64))[:, None, :]
    s = np.sin(ang.astype(np.float64))[:, None, :]
    x0 = x[..., :half].astype(np.float64)
    x1 = x[..., half:].astype(np.float64)
    out = np.empty_like(x)
    out[..., :half] = (x0 * c - x1 * s).astype(np.float32)
    out[..., half:] = (x0 * s + x1 * c).astype(np.float32)
    return round_to(out, dtype)


# ── silu * mul ───────────────────────────────────────────────────────────────

def silu_mul(gate: np.ndarray, up: np.ndarray, dtype: str) -> np.ndarray:
    """``out = silu(g) * u = g / (1 + exp(-g)) * u`` (silu_mul.cu:17-22), float64 math."""
    g = np.asarray(gate, np.float64)
    u = np.asarray(up, np.float64)
    with np.errstate(over="ignore"):
        out = g / (1.0 + np.exp(-g)) * u
    return round_to(out.astype(np.float32), dtype)


# ── tolerance helpers (the north-star parity bar) ───────────────────────────

def attention_paged(q: np.ndarray, k_pool: np.ndarray, v_pool: np.ndarray, block_table: np.ndarray, kv_len: int,
                    start_pos: int) -> np.ndarray:
    """The statement of ``paged_attention_kernel`` (``backends/fracture-cuda/kernels/attention_paged.cu:25-155``)
    in float64 for one sequence: ``q [N, Hq, d]`` (values), pools ``[rows, Hkv, d]`` (values) addressed by
    ``block_table[pos // 16] * 16 + pos % 16``; token t attends ``[0, min(start_pos + t + 1, kv_len))``
    (``:45-46``), Q head h reads KV head ``h // (Hq / Hkv)`` (``:42-43``); scores ``q . k / sqrt(d)``
    (``:54-76``), softmax (``:78-135``), ``sum p v`` (``:137-157``). A negative block-table entry
    leaves its positions out; a query with no position gives zeros."""
    q = np.asarray(q, np.float64)
    kp, vp = np.asarray(k_pool, np.float64), np.asarray(v_pool, np.float64)
    N, Hq, d = q.shape
    G = Hq // kp.shape[1]
    table = np.asarray(block_table, np.int64)
    out = np.zeros((N, Hq, d))
    for t in range(N):
        L = min(start_pos + t + 1, kv_len)
        pos = np.arange(L)
        blk = table[pos // 16]
        rows = (blk * 16 + pos % 16)[blk >= 0]
        if rows.size == 0:
            continue
        for h in range(Hq):
            k, v = kp[rows, h // G], vp[rows, h // G]
            s = k @ q[t, h] / np.sqrt(d)
            p = np.exp(s - s.max())
            out[t, h] = (p / p.sum()) @ v
    return out


def half_ulp(x: np.ndarray, dtype: str) -> np.ndarray:
    """Half a unit in the last place of the storage dtype at each value (its rounding bound)."""
    mant = {"f16": 10, "bf16": 7, "f32": 23}[dtype]
    ax = np.maximum(np.abs(np.asarray(x, np.float64)), 2.0 ** (-14 if dtype == "f16" else -126))
    return np.ldexp(1.0, np.floor(np.log2(ax)).astype(np.int64) - mant - 1)


def parity_report(actual: np.ndarray, expected: np.ndarray, dtype: str | None = None) -> dict:
    """max-abs error relative to the reference magnitude, and cosine similarity.

    With ``dtype``, each element's own storage rounding (half an ulp of that
    dtype at the expected value) is not counted as error: an output stored in
    BF16 cannot be closer than that to a float32 reference.
    """
    a = np.asarray(actual, np.float64).ravel()
    e = np.asarray(expected, np.float64).ravel()
    mag = float(np.max(np.abs(e))) if e.size else 0.0
    diff = np.abs(a - e)
    if dtype is not None and e.size:
        diff = np.maximum(diff - half_ulp(e, dtype), 0.0)
    err = float(np.max(diff)) if e.size else 0.0
    na, ne = float(np.linalg.norm(a)), float(np.linalg.norm(e))
    cos = float(np.dot(a, e) / (na * ne)) if na > 0 and ne > 0 else (1.0 if na == ne else 0.0)
    return {"max_abs": err, "rel_max_abs": err / mag if mag > 0 else err, "cosine": cos}


def assert_close_fp(actual, expected, rel=2e-3, min_cos=0.9999, label="", dtype=None):
    """North-star FP bar against a float32-or-better computation: max-abs error within
    ``rel`` x max|expected| beyond the output dtype's own rounding, and cosine >= ``min_cos``."""
    r = parity_report(actual, expected, dtype)
    assert r["rel_max_abs"] <= rel, f"{label}: max-abs {r['max_abs']:.3e} = {r['rel_max_abs']:.3e} of magnitude > {rel}"
    assert r["cosine"] >= min_cos, f"{label}: cosine {r['cosine']:.7f} < {min_cos}"
    return r


def compare_tensors(actual, expected, rtol: float, atol: float) -> int:
    """Mismatch count under the reference harness rule ``|a-e| <= atol + rtol*|e|``.

    ``tests/validation/src/tensor_compare.rs:226-292``.
    """
    a = np.asarray(actual, np.float32).ravel()
    e = np.asarray(expected, np.float32).ravel()
    return int(np.sum(np.abs(a - e) > atol + rtol * np.abs(e)))
