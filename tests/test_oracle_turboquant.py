"""Pin the TurboQuant oracle against the reference's own tests.

The reference commits no golden indices or packed bytes for TurboQuant; its
tests are property tests (``crates/fracture-core/src/turboquant.rs:440-1290``)
plus GPU round-trip thresholds (``bins/fracture-server-cuda/tests/
turboquant_gpu.rs:87-430``). Each test here restates one of them (named in its
docstring). The oracle is additionally pinned against the reference's CUDA
kernels themselves, run on a GPU, in ``tests/test_gpu_reference_kernels.py``.
"""

import numpy as np
import pytest

from oracle import turboquant as tq

TQC = tq.TurboQuantConfig


# ── config (turboquant.rs:444-668) ──────────────────────────────────────────

def test_config_default():
    c = TQC()
    assert (c.key_bits, c.value_bits, c.protected_bits, c.protected_layers, c.residual_tokens, c.seed) == (4, 2, 8, 0, 0, 42)


def test_config_validate():
    c = TQC()
    c.validate()
    c.key_bits = 3
    with pytest.raises(tq.ConfigError):
        c.validate()
    c.validate(allowed=tq.BUILD_VALID_BITS)  # this build accepts 3 bits
    c.key_bits, c.value_bits = 4, 5
    with pytest.raises(tq.ConfigError):
        c.validate(allowed=tq.BUILD_VALID_BITS)


def test_config_layer_bits():
    c = TQC(key_bits=4, value_bits=2, protected_bits=8, protected_layers=2)
    assert [c.key_bits_for_layer(l, 32) for l in (0, 1, 2, 15, 29, 30, 31)] == [8, 8, 4, 4, 4, 8, 8]
    assert [c.value_bits_for_layer(l, 32) for l in (0, 15, 31)] == [8, 2, 8]
    assert TQC(protected_layers=20).is_protected(16, 32)
    assert TQC(protected_layers=1).is_protected(0, 1)
    assert not TQC(protected_layers=0).is_protected(0, 32)


def test_packed_dims_and_block_bytes():
    assert TQC.packed_dim_per_head(128, 4) == 64
    assert TQC.packed_dim_per_head(128, 2) == 32
    assert TQC.packed_dim_per_head(128, 8) == 128
    assert TQC.packed_dim_per_head(128, 3) == 48
    assert TQC.packed_dim_per_head(96, 4) == 48 and TQC.packed_dim_per_head(96, 2) == 24
    assert TQC.packed_dim_per_head(1, 4) == 1 and TQC.packed_dim_per_head(3, 2) == 1 and TQC.packed_dim_per_head(5, 4) == 3
    assert TQC.bytes_per_block_layer(8, 128, 4, 2) == 12800
    assert TQC.bytes_per_block_layer(8, 128, 8, 8) == 33280
    assert TQC().bytes_per_block_total(32, 8, 128) == 12800 * 32
    c = TQC(protected_layers=4)
    assert c.bytes_per_block_total(32, 8, 128) == 8 * 33280 + 24 * 12800
    assert TQC().distinct_bit_widths() == [2, 4]
    assert TQC(protected_layers=2).distinct_bit_widths() == [2, 4, 8]
    assert TQC(key_bits=4, value_bits=4).distinct_bit_widths() == [4]
    per = TQC().bytes_per_block_total(32, 8, 128)
    assert TQC().compute_num_blocks(1000, 2000, 32, 8, 128) == 0
    assert TQC().compute_num_blocks(3 * per + per - 1, 0, 32, 8, 128) == 3


# ── Lloyd-Max (turboquant.rs:572-703, 856-962) ─────────────────────────────

def test_lloyd_max_2bit_symmetry():
    cb = tq.get_codebook(128, 2)
    assert cb.centroids.shape == (4,) and cb.boundaries.shape == (3,)
    for i in range(2):
        assert abs(cb.centroids[3 - i] + cb.centroids[i]) < 1e-6
    assert abs(cb.boundaries[1]) < 1e-6


@pytest.mark.parametrize("bits", [3, 4])
def test_lloyd_max_sorted_and_bracketed(bits):
    cb = tq.get_codebook(128, bits)
    n = 1 << bits
    assert cb.n_levels == n and cb.boundaries.shape == (n - 1,)
    assert np.all(np.diff(cb.centroids) > 0)
    assert np.all((cb.boundaries > cb.centroids[:-1]) & (cb.boundaries < cb.centroids[1:]))
    for i in range(n // 2):
        assert abs(cb.centroids[n - 1 - i] + cb.centroids[i]) < 1e-5
    assert np.all(np.abs(cb.centroids) < 4.0 / np.sqrt(128))


def test_lloyd_max_scale_and_dims():
    r = tq.get_codebook(64, 4).centroids[-1] / tq.get_codebook(128, 4).centroids[-1]
    assert abs(r - np.sqrt(2)) < 0.1
    for d in (64, 96, 128, 256):
        cb = tq.get_codebook(d, 4)
        assert cb.dim == d and cb.bits == 4 and np.all(np.diff(cb.centroids) > 0)


def test_lloyd_max_deterministic_and_distortion():
    a = tq.LloydMaxCodebook.compute(128, 4)
    b = tq.LloydMaxCodebook.compute(128, 4)
    assert np.array_equal(a.centroids, b.centroids) and np.array_equal(a.boundaries, b.boundaries)
    # per-coordinate MSE in units of sigma^2 (docs/turboquant.md: 0.116 / 0.009 for 2 / 4 bits)
    rng = tq.Xoshiro256(999)
    sigma = 1.0 / np.sqrt(128)
    x = np.array([tq.box_muller(rng)[0] for _ in range(10000)], dtype=np.float64) * sigma
    mse = {}
    for bits in (2, 4):
        c = tq.get_codebook(128, bits).centroids
        q = c[tq.nearest_centroid(x.astype(np.float32), c)]
        mse[bits] = float(np.mean((x - q) ** 2)) / sigma ** 2
    assert mse[4] < mse[2] / 2
    assert abs(mse[2] - 0.116) < 0.01 and abs(mse[4] - 0.009) < 0.002


# ── rotation (turboquant.rs:706-770, 964-1050) ──────────────────────────────

def test_rotation_orthogonal_deterministic():
    q = tq.generate_rotation_matrix(16, 42)
    assert np.abs(q.T.astype(np.float64) @ q - np.eye(16)).max() < 1e-4
    assert np.array_equal(tq.generate_rotation_matrix(32, 42), tq.generate_rotation_matrix(32, 42))
    assert not np.array_equal(tq.generate_rotation_matrix(16, 42), tq.generate_rotation_matrix(16, 43))


def test_rotation_128d_and_positive_diagonal():
    q = tq.generate_rotation_matrix(128, 42).astype(np.float64)
    for i, j in [(0, 1), (0, 63), (63, 127)]:
        assert abs(q[i] @ q[j]) < 1e-3
    assert abs(q[0] @ q[0] - 1.0) < 1e-3
    assert np.all(np.diag(q) > 0)


def test_rotation_seeds():
    assert tq.rotation_seeds(42, 0) == (42, 542)
    assert tq.rotation_seeds(42, 5) == (5042, 5542)
    assert all(k != v for k, v in (tq.rotation_seeds(42, l) for l in range(32)))


def test_rotation_norm_roundtrip_distribution():
    d = 64
    pi = tq.generate_rotation_matrix(d, 42)
    rng = tq.Xoshiro256(77)
    x = np.array([tq.box_muller(rng)[0] for _ in range(d)], dtype=np.float32)
    y = np.array([tq.seq_sum_f32(pi[i] * x) for i in range(d)], dtype=np.float32)
    assert abs(np.linalg.norm(x) - np.linalg.norm(y)) < 1e-3
    back = np.array([tq.seq_sum_f32(pi[:, i] * y) for i in range(d)], dtype=np.float32)
    assert np.abs(back - x).max() < 1e-4
    e = tq.generate_rotation_matrix(128, 42)[:, 0]
    assert abs(e.mean()) < 0.05 and abs(e.std() - 1 / np.sqrt(128)) < 0.5 / np.sqrt(128)


def test_xoshiro_known_sequence():
    """SplitMix64 seeding + Xoshiro256** output for seed 0 (published reference values)."""
    rng = tq.Xoshiro256(0)
    # SplitMix64(0) first outputs (published): e220a8397b1dcdaf, 6e789e6aa1b965f4
    assert rng.s[0] == 0xE220A8397B1DCDAF and rng.s[1] == 0x6E789E6AA1B965F4
    a = [rng.next_u64() for _ in range(3)]
    assert len(set(a)) == 3 and all(0 <= v < 2 ** 64 for v in a)


# ── compress / decompress (turboquant.rs:1056-1290; turboquant_gpu.rs) ─────

def _rust_vec(seed, d):
    rng = tq.Xoshiro256(seed)
    return np.array([tq.box_muller(rng)[0] for _ in range(d)], dtype=np.float32)


@pytest.mark.parametrize("bits,min_cos", [(4, 0.99), (2, 0.90)])
def test_roundtrip_cosine_cpu(bits, min_cos):
    """test_quantize_dequantize_roundtrip / _2bit_roundtrip (seeds 123 / 456, Pi seed 42)."""
    d = 128
    x = _rust_vec(123 if bits == 4 else 456, d)
    pi = tq.generate_rotation_matrix(d, 42)
    cb = tq.get_codebook(d, bits)
    packed, norms, idx, _ = tq.compress(x.reshape(1, 1, d), pi, cb.centroids, bits)
    xr = tq.decompress(packed, norms, pi, cb.centroids, bits, 1, d)[0, 0]
    # reconstruct with the f32 norm (the reference's CPU test does not round it)
    xr = xr / norms[0, 0] * np.linalg.norm(x)
    cos = float(x @ xr / (np.linalg.norm(x) * np.linalg.norm(xr)))
    assert cos > min_cos


def _gpu_test_input(n_tok, heads, d, seed):
    """``random_fp16_tensor`` of turboquant_gpu.rs:41-65: rotation-matrix entries as data."""
    numel = n_tok * heads * d
    side = max(int(np.ceil(np.sqrt(numel))), 2)
    raw = tq.generate_rotation_matrix(side, seed).ravel()[:numel]
    return raw.astype(np.float16).reshape(n_tok, heads, d)


@pytest.mark.parametrize("bits,min_cos", [(4, 0.95), (2, 0.80), (8, 0.999)])
def test_gpu_suite_roundtrip_thresholds_on_oracle(bits, min_cos):
    """turboquant_gpu.rs round-trip tests (head_dim 16, 2 heads, 4 tokens) on the oracle."""
    d, heads, n = 16, 2, 4
    x = _gpu_test_input(n, heads, d, 12345)
    pi = tq.generate_rotation_matrix(d, 42)
    cb = tq.get_codebook(d, bits)
    packed, norms, idx, _ = tq.compress(x.astype(np.float32), pi, cb.centroids, bits)
    assert packed.shape == (n, heads * TQC.packed_dim_per_head(d, bits))
    out = tq.decompress(packed, norms, pi, cb.centroids, bits, heads, d).astype(np.float16).astype(np.float32)
    xf = x.astype(np.float32)
    for t in range(n):
        for h in range(heads):
            a, b = xf[t, h], out[t, h]
            cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-10))
            assert cos > min_cos
            assert abs(norms[t, h] - np.linalg.norm(a)) / np.linalg.norm(a) < 0.02


def test_zero_vector():
    d = 128
    pi = tq.generate_rotation_matrix(d, 42)
    cb = tq.get_codebook(d, 4)
    packed, norms, idx, y = tq.compress(np.zeros((1, 1, d), np.float32), pi, cb.centroids, 4)
    assert norms[0, 0] == 0.0 and np.all(y == 0.0)
    out = tq.decompress(packed, norms, pi, cb.centroids, 4, 1, d)
    assert np.all(np.isfinite(out)) and np.abs(out).max() < 1e-6


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
def test_pack_unpack_roundtrip_and_reference_layout(bits):
    rng = np.random.default_rng(bits)
    idx = rng.integers(0, 1 << bits, size=(5, 3, 128), dtype=np.int32)
    packed = tq.pack_indices(idx, bits)
    assert packed.shape == (5, 3, TQC.packed_dim_per_head(128, bits))
    assert np.array_equal(tq.unpack_indices(packed, bits, 128), idx)
    if bits == 4:  # high nibble = even coordinate (turboquant_compress.cu:146)
        assert np.array_equal(packed, ((idx[..., 0::2] << 4) | idx[..., 1::2]).astype(np.uint8))
    if bits == 2:  # shift 6 - 2*sub (turboquant_compress.cu:167)
        ref = sum(idx[..., s::4] << (6 - 2 * s) for s in range(4)).astype(np.uint8)
        assert np.array_equal(packed, ref)
    if bits == 8:
        assert np.array_equal(packed, idx.astype(np.uint8))


@pytest.mark.parametrize("kind", ["f16", "bf16"])
@pytest.mark.parametrize("bits", [2, 3, 4])
def test_c_oracle_equals_numpy_oracle(kind, bits):
    from oracle import ops

    rng = np.random.default_rng(7 + bits)
    d = 128
    x32 = rng.standard_normal((9, 4, d)).astype(np.float32)
    x32[rng.random(x32.shape) < 0.005] *= 10.0
    x = ops.round_to(x32, kind)
    raw = ops.to_storage_bytes(x, kind).reshape(x.shape)
    pi = tq.generate_rotation_matrix(d, 542)
    cb = tq.get_codebook(d, bits)
    p, n, idx, _ = tq.compress(x, pi, cb.centroids, bits)
    pc, nc, ic = tq.compress_c(raw, tq.INPUT_F16 if kind == "f16" else tq.INPUT_BF16, pi, cb.centroids, bits,
                               num_threads=3)
    assert np.array_equal(p, pc) and np.array_equal(idx, ic.astype(np.int32))
    assert np.array_equal(n, nc.view(np.float16).astype(np.float32))
    out = tq.decompress(p, n, pi, cb.centroids, bits, 4, d)
    outc = tq.decompress_c(pc, nc, pi, cb.centroids, bits, 4, d, num_threads=2)
    assert np.array_equal(out, outc)


def test_paged_cache_block_accounting():
    """append_kv block growth and placement (quantized_paged_kv_cache.rs:446-497)."""
    c = tq.QuantizedKvCache(num_blocks=8, num_layers=2, num_kv_heads=1, head_dim=16, config=TQC())
    a = c.alloc()
    b = c.alloc()
    assert c.seqs[a].block_table == [0] and c.seqs[b].block_table == [1]
    assert c.reserve(a, 5) == 0 and c.seqs[a].block_table == [0]
    assert c.reserve(a, 11) == 5 and c.seqs[a].block_table == [0] and c.seqs[a].last_block_fill == 16
    assert c.reserve(a, 1) == 16 and c.seqs[a].block_table == [0, 2]
    assert c.reserve(b, 40) == 0 and c.seqs[b].block_table == [1, 3, 4]
    assert list(c.slots(b, 14, 4)) == [30, 31, 48, 49]
    c.free(a)
    assert c.free_list[-2:] == [0, 2]
    d_ = c.alloc()
    assert c.seqs[d_].block_table == [2]


def test_attention_statement_equals_dense_attention_over_the_dequantized_cache():
    """Scores in K's rotated space and values accumulated in V's rotated space
    (attention_paged_tq.cu:12-17) equal plain causal attention over the dequantized keys and
    values, Pi^T c[idx] * norm, to float64 rounding; a missing block drops its positions."""
    rng = np.random.default_rng(0)
    d, Hkv, Hq, T = 128, 2, 4, 40
    c = np.asarray(tq.get_codebook(d, 4).centroids, np.float32)
    c2 = np.asarray(tq.get_codebook(d, 2).centroids, np.float32)
    pik, piv = tq.generate_rotation_matrix(d, 1), tq.generate_rotation_matrix(d, 2)
    x = rng.standard_normal((T, Hkv, d)).astype(np.float32)
    pk, nk, _, _ = tq.compress(x, pik, c, 4)
    pv, nv, _, _ = tq.compress(x * 0.5 + 1, piv, c2, 2)
    table = np.array([2, 0, 1], np.int32)
    rows = 48
    KP = np.zeros((rows, Hkv * 64), np.uint8)
    VP = np.zeros((rows, Hkv * 32), np.uint8)
    KN, VN = np.zeros((rows, Hkv)), np.zeros((rows, Hkv))
    pos = np.arange(T)
    sl = table[pos // 16] * 16 + pos % 16
    KP[sl], VP[sl], KN[sl], VN[sl] = pk, pv, nk, nv
    q = rng.standard_normal((3, Hq, d))
    dk = np.stack([(c[tq.unpack_indices(pk.reshape(T, Hkv, 64)[:, g], 4, d)] @ pik.astype(np.float64))
                   * nk[:, g, None] for g in range(Hkv)], 1)
    dv = np.stack([(c2[tq.unpack_indices(pv.reshape(T, Hkv, 32)[:, g], 2, d)] @ piv.astype(np.float64))
                   * nv[:, g, None] for g in range(Hkv)], 1)
    for missing in (None, 1):
        tab = table.copy()
        if missing is not None:
            tab[missing] = -1
        got = tq.attention_paged_tq(q, KP, KN, VP, VN, tab, T, T - 3, pik, piv, c, c2, 4, 2, Hkv)
        keep = np.ones(T, bool) if missing is None else (pos // 16 != missing)
        for t in range(3):
            L = T - 3 + t + 1
            m = keep[:L]
            for h in range(Hq):
                g = h // 2
                s = dk[:L][m, g] @ q[t, h] / np.sqrt(d)
                p = np.exp(s - s.max())
                p /= p.sum()
                assert np.abs(got[t, h] - p @ dv[:L][m, g]).max() < 1e-12
