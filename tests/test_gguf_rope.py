"""RoPE frequencies read from GGUF model files (fb_gguf_rope_params / fb_rope_freqs_from_gguf).

The reference reads only `{arch}.rope.freq_base` (crates/fracture-gguf/src/parser.rs:482) and
builds its table with precompute_rope_freqs(head_dim, theta) (bins/fracture-server-cuda/src/
main.rs:104). These tests write GGUF files with the `gguf` package (0.19, the writer llama.cpp's
converters use) carrying the three forms Llama 3.1 scaling takes in the wild, and check the table
against the CPU statement: the reference's table, the published llama3 rule
(oracle.ops.rope_freqs_llama3, itself pinned to transformers' "llama3" rope init), and the
per-pair divisor tensor. Host code only: no GPU."""

import math

import numpy as np
import pytest

gguf = pytest.importorskip("gguf")

from fracture_b200 import kernels as K  # noqa: E402
from oracle import ops  # noqa: E402

HD, THETA = 128, 500000.0


def write(path, arch="llama", kv=None, rope_factors=None, extra_tensor=True):
    w = gguf.GGUFWriter(str(path), arch)
    w.add_uint32(f"{arch}.rope.dimension_count", HD)
    w.add_float32(f"{arch}.rope.freq_base", THETA)
    w.add_array(f"{arch}.some_array", [1, 2, 3])  # values of every kind before and after
    w.add_string("general.name", "test")
    for key, (kind, val) in (kv or {}).items():
        getattr(w, f"add_{kind}")(key, val)
    if extra_tensor:
        w.add_tensor("token_embd.weight", np.arange(6 * 4, dtype=np.float32).reshape(6, 4))
    if rope_factors is not None:
        w.add_tensor("rope_freqs.weight", np.asarray(rope_factors, dtype=np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def llama3_divisors(factor=8.0, low=1.0, high=4.0, orig=8192):
    """Per-pair divisors of the llama3 rule, as a converter computes them from the base table."""
    base = ops.rope_freqs(HD, THETA).astype(np.float64)
    out = []
    for f in base:
        wavelen = 2 * math.pi / f
        if wavelen < orig / high:
            out.append(1.0)
        elif wavelen > orig / low:
            out.append(factor)
        else:
            s = (orig / wavelen - low) / (high - low)
            out.append(1.0 / ((1 - s) / factor + s))
    return np.array(out, dtype=np.float32)


def test_freq_base_only_equals_the_reference_table(tmp_path):
    p = tmp_path / "plain.gguf"
    write(p)
    params = K.gguf_rope_params(p)
    assert params["scaling"] == "none" and params["theta"] == THETA and params["head_dim"] == HD
    assert np.array_equal(K.rope_freqs_from_gguf(p, HD), ops.rope_freqs(HD, THETA))


def test_llama3_metadata(tmp_path):
    p = tmp_path / "llama3.gguf"
    write(p, kv={"llama.rope.scaling.type": ("string", "llama3"), "llama.rope.scaling.factor": ("float32", 8.0),
                 "llama.rope.scaling.original_context_length": ("uint32", 8192),
                 "llama.rope.scaling.low_freq_factor": ("float32", 1.0),
                 "llama.rope.scaling.high_freq_factor": ("float32", 4.0)})
    params = K.gguf_rope_params(p)
    assert params["scaling"] == "llama3" and params["factor"] == 8.0 and params["original_context"] == 8192
    assert np.array_equal(K.rope_freqs_from_gguf(p, HD), ops.rope_freqs_llama3(HD, THETA, 8.0, 1.0, 4.0, 8192))


def test_llama3_metadata_defaults_for_the_frequency_factors(tmp_path):
    """A file with type/factor/original context but no low/high factors gets Llama 3.1's 1 and 4."""
    p = tmp_path / "llama3_short.gguf"
    write(p, kv={"llama.rope.scaling.type": ("string", "llama3"), "llama.rope.scaling.factor": ("float32", 8.0),
                 "llama.rope.scaling.original_context_length": ("uint32", 8192)})
    assert np.array_equal(K.rope_freqs_from_gguf(p, HD), ops.rope_freqs_llama3(HD, THETA, 8.0, 1.0, 4.0, 8192))


def test_rope_freqs_tensor_of_divisors(tmp_path):
    """llama.cpp's converter writes the llama3 scaling as a rope_freqs tensor of per-pair divisors
    (after other tensors, so its data offset is not zero); the table is base / divisor and agrees
    with the llama3 rule to float32 rounding."""
    p = tmp_path / "factors.gguf"
    div = llama3_divisors()
    write(p, rope_factors=div)
    params = K.gguf_rope_params(p)
    assert params["scaling"] == "factors" and params["num_freq_factors"] == HD // 2
    got = K.rope_freqs_from_gguf(p, HD)
    assert np.array_equal(got, (ops.rope_freqs(HD, THETA) / div).astype(np.float32))
    np.testing.assert_allclose(got, ops.rope_freqs_llama3(HD, THETA, 8.0, 1.0, 4.0, 8192), rtol=3e-7)


def test_linear_scaling_and_other_architecture(tmp_path):
    p = tmp_path / "linear.gguf"
    write(p, arch="qwen2", kv={"qwen2.rope.scaling.type": ("string", "linear"),
                               "qwen2.rope.scaling.factor": ("float32", 4.0)})
    params = K.gguf_rope_params(p)
    assert params["scaling"] == "linear"
    assert np.array_equal(K.rope_freqs_from_gguf(p, HD),
                          (ops.rope_freqs(HD, THETA).astype(np.float64) / 4.0).astype(np.float32))


def test_errors_are_reported(tmp_path):
    with pytest.raises(ValueError, match="cannot open"):
        K.rope_freqs_from_gguf(tmp_path / "missing.gguf", HD)
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + b"\0" * 64)
    with pytest.raises(ValueError, match="bad magic"):
        K.gguf_rope_params(bad)
    p = tmp_path / "short.gguf"
    write(p, rope_factors=np.ones(10, np.float32))
    with pytest.raises(ValueError, match="head_dim/2"):
        K.rope_freqs_from_gguf(p, HD)
