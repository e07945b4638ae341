"""Pin the elementwise oracle against the reference's committed fixture goldens.

The goldens (``tests/golden/fixture_prompt{0,1}.npz``, extracted by
``tests/golden/make_golden.py``) are the reference's own per-layer dumps of the
tiny seeded Llama (``tests/reference-fixture`` in the Fracture repository).
Tolerances are the reference harness's (``tests/model-validation/tests/
kernels.rs:118-123`` RTOL=ATOL=1e-3, LOOSE 5e-3 for norms; RoPE rtol 0.01 /
atol 0.025 at ``:1551-1552``), and where the oracle reproduces a golden exactly
the test asserts that.
"""

import json

import numpy as np
import pytest

from oracle import ops

RTOL = ATOL = 1e-3
LOOSE = 5e-3


def _meta(z):
    return json.loads(bytes(z["meta_json"]))


@pytest.mark.parametrize("p", [0, 1])
def test_embedding_bit_exact(golden, p):
    z = golden[p]
    if "embeddings" not in z.files:
        pytest.skip("prompt has no embeddings dump")
    out = ops.embedding(z["token_embd"].astype(np.float32), z["token_ids"].astype(np.uint32))
    assert np.array_equal(out, z["embeddings"])


def test_embedding_oov_rows_are_zero():
    table = np.arange(12, dtype=np.float32).reshape(3, 4) + 1
    out = ops.embedding(table, np.array([0, 3, 2, 0xFFFFFFFF], dtype=np.uint32))
    assert np.array_equal(out[0], table[0]) and np.array_equal(out[2], table[2])
    assert not out[1].any() and not out[3].any()


@pytest.mark.parametrize("p", [0, 1])
@pytest.mark.parametrize("layer", range(4))
def test_rmsnorm_attn(golden, p, layer):
    z = golden[p]
    m = _meta(z)
    out = ops.rmsnorm(z[f"l{layer}.input_hidden"], z[f"l{layer}.attn_norm_w"].astype(np.float32),
                      m["rms_norm_eps"], "f16")
    ref = z[f"l{layer}.post_attn_norm"]
    assert ops.compare_tensors(out, ref, LOOSE, LOOSE) == 0
    # The oracle's single-rounding form reproduces the dump except for rare 1-ulp ties.
    assert np.mean(out != ref) < 1e-3


@pytest.mark.parametrize("p", [0, 1])
@pytest.mark.parametrize("layer", range(4))
def test_fused_residual_add_rmsnorm(golden, p, layer):
    """output_hidden = post_attn_residual + ffn_output (bit-exact), ffn norm pinned too."""
    z = golden[p]
    m = _meta(z)
    w = z[f"l{layer}.ffn_norm_w"].astype(np.float32)
    h, _ = ops.add_rmsnorm(z[f"l{layer}.post_attn_residual"], z[f"l{layer}.ffn_output"], w,
                           m["rms_norm_eps"], "f16")
    assert np.array_equal(h, z[f"l{layer}.output_hidden"])
    n = ops.rmsnorm(z[f"l{layer}.post_attn_residual"], w, m["rms_norm_eps"], "f16")
    assert ops.compare_tensors(n, z[f"l{layer}.post_ffn_norm"], LOOSE, LOOSE) == 0
    if layer + 1 < m["num_layers"]:
        # next layer's input is this layer's output: the chain add -> norm is consistent
        assert np.array_equal(h, z[f"l{layer + 1}.input_hidden"])


@pytest.mark.parametrize("p", [0, 1])
@pytest.mark.parametrize("layer", range(4))
def test_rope_unscaled(golden, p, layer):
    z = golden[p]
    m = _meta(z)
    T = z[f"l{layer}.q"].shape[0]
    hd = m["head_dim"]
    f = ops.rope_freqs(hd, m["rope_theta"])
    q = z[f"l{layer}.q"].reshape(T, m["num_q_heads"], hd)
    k = z[f"l{layer}.k"].reshape(T, m["num_kv_heads"], hd)
    qr = ops.rope(q, np.arange(T), f, "f32")
    kr = ops.rope(k, np.arange(T), f, "f32")
    # the dump is float32 (not rounded to fp16): the oracle agrees to ~1e-5 absolute
    assert np.abs(qr - z[f"l{layer}.q_rope"]).max() < 1e-4
    assert np.abs(kr - z[f"l{layer}.k_rope"]).max() < 1e-4
    assert ops.compare_tensors(ops.round_to(qr, "f16"), z[f"l{layer}.q_rope"], 0.01, 0.025) == 0


@pytest.mark.parametrize("p", [0, 1])
@pytest.mark.parametrize("layer", range(4))
def test_silu_mul(golden, p, layer):
    z = golden[p]
    if f"l{layer}.silu_mul" not in z.files:
        pytest.skip("prompt has no silu_mul dump for this layer")
    out = ops.silu_mul(z[f"l{layer}.gate"], z[f"l{layer}.up"], "f16")
    ref = z[f"l{layer}.silu_mul"]
    assert ops.compare_tensors(out, ref, RTOL, ATOL) == 0
    ops.assert_close_fp(out, ref, label="silu_mul")


def test_rope_freqs_match_reference_formula():
    """``precompute_rope_freqs``: f64 power cast to f32, then an f32 reciprocal (src/lib.rs:133-138)."""
    f = ops.rope_freqs(128, 500000.0)
    assert f.dtype == np.float32 and f.shape == (64,)
    assert f[0] == np.float32(1.0)
    i = 17
    assert f[i] == np.float32(1.0) / np.float32(500000.0 ** (2.0 * i / 128.0))
    # the reference's own test pins the extreme values (backends/fracture-cuda/src/tests.rs:2402)
    assert abs(float(f[-1]) - 1.0 / 500000.0 ** (126.0 / 128.0)) < 1e-9


def test_llama3_freqs_match_transformers():
    """The llama3 rule has no reference implementation: check against transformers at run time."""
    torch = pytest.importorskip("torch")
    tr = pytest.importorskip("transformers")
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS

    cfg = tr.LlamaConfig(hidden_size=4096, num_attention_heads=32, num_key_value_heads=8,
                         max_position_embeddings=131072,
                         rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                       "high_freq_factor": 4.0, "original_max_position_embeddings": 8192,
                                       "rope_theta": 500000.0},
                         rope_theta=500000.0)
    inv_freq, _ = ROPE_INIT_FUNCTIONS["llama3"](cfg, torch.device("cpu"))
    ours = ops.rope_freqs_llama3(128, 500000.0, 8.0, 1.0, 4.0, 8192)
    ref = inv_freq.to(torch.float64).numpy()
    # transformers builds the base frequencies in float32 arithmetic; the reference
    # builds them in f64 -> f32: they agree to a few float32 ulps.
    np.testing.assert_allclose(ours, ref, rtol=2e-6, atol=0)
    # the three regimes are all present at Llama-3.1 parameters
    base = ops.rope_freqs(128, 500000.0)
    assert ours[0] == base[0] and ours[-1] == np.float32(base[-1] / 8.0)
    assert np.any((ours != base) & (ours != (base / 8.0).astype(np.float32)))


def test_compare_tensors_rule():
    assert ops.compare_tensors([1.0, 2.0], [1.0, 2.0005], 1e-3, 1e-3) == 0
    assert ops.compare_tensors([1.0, 2.1], [1.0, 2.0], 1e-3, 1e-3) == 1


def test_round_to_bf16_nearest_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 3.0e38], dtype=np.float32)
    r = ops.round_to(x, "bf16")
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == np.float32(1.0 + 4 * 2 ** -8) and r[3] == -2.5
    import torch

    t = torch.tensor(x).to(torch.bfloat16).to(torch.float32).numpy()
    assert np.array_equal(r, t)
