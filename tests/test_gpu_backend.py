"""The Backend-trait mirror over the C ABI, read like the reference's backend tests
(backends/fracture-cuda/src/tests.rs): allocation, copies, error variants and
messages, the deferred add fused into rmsnorm, rope tables, timers, and the
quantized paged KV cache (crates/fracture-engine/src/quantized_paged_kv_cache.rs)."""

import numpy as np
import pytest

from fracture_b200.backend import (FB_BF16, FB_FP16, FB_FP32, FB_INT8, BackendError, CudaBackend, InvalidShape,
                                   ModelConfigError,
                                   KvCacheError, OutOfMemory, PagedKvCache, QuantizedKvCache, TensorNotFound, TurboQuantConfig)
from fracture_b200 import kernels as K
from oracle import ops, turboquant as tq

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    b = CudaBackend(0)
    yield b
    b.close()


def upload(be, x, dt=FB_FP16):
    x = np.asarray(x, np.float32)
    t = be.alloc(x.shape, dt)
    npdt = {FB_FP16: "f16", FB_BF16: "bf16", FB_FP32: "f32"}[dt]
    be.copy_to_device(t, ops.to_storage_bytes(ops.round_to(x, npdt), npdt))
    return t


def download(be, t):
    raw = be.copy_to_host(t)
    if t.dtype == FB_FP16:
        return raw.view(np.float16).astype(np.float32).reshape(t.shape)
    if t.dtype == FB_BF16:
        return ops.bf16_bits_to_f32(raw.view(np.uint16)).reshape(t.shape)
    return raw.view(np.float32).reshape(t.shape)


def test_alloc_free_copy_roundtrip(be):
    t = be.alloc([4, 8], FB_FP16)
    x = np.arange(32, dtype=np.float16).reshape(4, 8)
    be.copy_to_device(t, x)
    assert np.array_equal(download(be, t), x.astype(np.float32))
    be.free(t)
    with pytest.raises(TensorNotFound, match=f"tensor id {t.id}"):
        be.free(t)  # double free (tests.rs:488)
    with pytest.raises(TensorNotFound):
        be.copy_to_host(t)  # use after free (tests.rs:496)
    assert "B200" in be.device_name() or be.device_name()
    assert be.total_memory() > be.available_memory() > 0


def test_copy_buffer_too_small_messages(be):
    t = be.alloc([16], FB_FP32)
    with pytest.raises(InvalidShape, match="source buffer too small: 8 < 64"):
        be.copy_to_device(t, np.zeros(2, np.float32))
    with pytest.raises(InvalidShape, match="destination buffer too small"):
        be.copy_to_host(t, np.zeros(3, np.float32))
    be.free(t)


def test_alloc_huge_fails_with_backend_error(be):
    with pytest.raises(BackendError, match="CUDA error"):
        be.alloc([1 << 50], FB_FP32)


def test_int4_and_int8_sizes(be):
    t = be.alloc([1023], 4)
    assert t.size_bytes() == 512
    be.free(t)
    t = be.alloc([16, 64], FB_INT8)
    assert t.size_bytes() == 1024
    be.free(t)


@pytest.mark.parametrize("dt", [FB_FP16, FB_BF16])
def test_add_then_rmsnorm_fuses_and_matches_separate_ops(be, dt):
    npdt = "f16" if dt == FB_FP16 else "bf16"
    rng = np.random.default_rng(0)
    rows, cols = 24, 4096
    h0 = ops.round_to(rng.standard_normal((rows, cols)) * 3, npdt)
    r = ops.round_to(rng.standard_normal((rows, cols)), npdt)
    w = ops.round_to(1 + 0.02 * rng.standard_normal(cols), npdt)
    th, tr, tw, tn = upload(be, h0, dt), upload(be, r, dt), upload(be, w, dt), be.alloc([rows, cols], dt)
    be.add(th, tr, th)  # deferred
    be.rmsnorm(th, tw, 1e-5, tn)  # fused launch
    h_ref, _ = ops.add_rmsnorm(h0, r, w, 1e-5, npdt)
    assert np.array_equal(download(be, th), h_ref)
    ops.assert_close_fp(download(be, tn), ops.rmsnorm(h_ref, w, 1e-5, "f32"), dtype=npdt)
    # a pending add is flushed by any other use of the tensor
    be.add(th, tr, th)
    got = download(be, th)  # copy_to_host flushes
    assert np.array_equal(got, ops.add(h_ref, r, npdt))
    be.add(th, tr, th)
    be.silu_mul(th, tr, tn)  # flushes, then silu
    h2 = ops.add(ops.add(h_ref, r, npdt), r, npdt)
    ops.assert_close_fp(download(be, tn), ops.silu_mul(h2, r, "f32"), dtype=npdt)
    for t in (th, tr, tw, tn):
        be.free(t)


def test_shape_errors(be):
    a, b = be.alloc([4, 8], FB_FP16), be.alloc([4, 9], FB_FP16)
    with pytest.raises(InvalidShape, match=r"add: a shape \[4, 8\] != b shape \[4, 9\]"):
        be.add(a, b, a)
    with pytest.raises(InvalidShape, match="silu_mul: gate shape"):
        be.silu_mul(a, b, a)
    with pytest.raises(InvalidShape, match="copy_rows: src_offset"):
        be.copy_rows(a, a, 3, 0, 2)
    with pytest.raises(InvalidShape, match="copy_rows: dst_offset"):
        be.copy_rows(a, a, 0, 3, 2)
    with pytest.raises(InvalidShape, match="column shape"):
        be.copy_rows(a, b, 0, 0, 1)
    be.free(a)
    be.free(b)


def test_copy_rows(be):
    x = np.arange(6 * 4, dtype=np.float32).reshape(6, 4)
    s, d = upload(be, x), be.alloc([5, 4], FB_FP16)
    be.copy_to_device(d, np.zeros((5, 4), np.float16))
    be.copy_rows(s, d, 2, 1, 3)
    got = download(be, d)
    assert np.array_equal(got[1:4], x[2:5]) and not got[0].any() and not got[4].any()


def test_rope_requires_freq_table_then_matches_oracle():
    b = CudaBackend(0)
    q, k = upload(b, np.ones((2, 4, 32))), upload(b, np.ones((2, 2, 32)))
    with pytest.raises(BackendError, match="RoPE frequency table not initialized"):
        b.rope(q, k, [0, 1], 5e5, 32)
    b.precompute_rope_freqs_llama3(128, 5e5, 8.0, 1.0, 4.0, 8192)
    rng = np.random.default_rng(1)
    T = 64
    qx = ops.round_to(rng.standard_normal((T, 32, 128)), "bf16")
    kx = ops.round_to(rng.standard_normal((T, 8, 128)), "bf16")
    pos = rng.integers(0, 8192, T).astype(np.uint32)
    tq_, tk = upload(b, qx, FB_BF16), upload(b, kx, FB_BF16)
    for _ in range(3):  # same positions every layer: uploaded once, reused
        b.rope(tq_, tk, pos, 5e5, 128)
    f = ops.rope_freqs_llama3(128, 5e5, 8.0, 1.0, 4.0, 8192)
    ref_q, ref_k = qx, kx
    for _ in range(3):
        ref_q, ref_k = ops.rope(ref_q, pos, f, "bf16"), ops.rope(ref_k, pos, f, "bf16")
    ops.assert_close_fp(download(b, tq_), ref_q, rel=6e-3, dtype="bf16")
    ops.assert_close_fp(download(b, tk), ref_k, rel=6e-3, dtype="bf16")
    b.close()


def test_rope_table_from_a_gguf_file(tmp_path):
    """precompute_rope_freqs_gguf: a GGUF file whose metadata says llama3 scaling gives the same
    rotated Q/K bytes as precompute_rope_freqs_llama3 with those parameters (the call-site change
    for bins/fracture-server-cuda/src/main.rs:104)."""
    gguf = pytest.importorskip("gguf")
    path = tmp_path / "llama31.gguf"
    w = gguf.GGUFWriter(str(path), "llama")
    w.add_float32("llama.rope.freq_base", 5e5)
    w.add_string("llama.rope.scaling.type", "llama3")
    w.add_float32("llama.rope.scaling.factor", 8.0)
    w.add_uint32("llama.rope.scaling.original_context_length", 8192)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    rng = np.random.default_rng(5)
    qx = ops.round_to(rng.standard_normal((16, 32, 128)), "f16")
    kx = ops.round_to(rng.standard_normal((16, 8, 128)), "f16")
    pos = rng.integers(0, 8192, 16).astype(np.uint32)
    outs = []
    for how in ("gguf", "params"):
        b = CudaBackend(0)
        if how == "gguf":
            b.precompute_rope_freqs_gguf(128, path)
        else:
            b.precompute_rope_freqs_llama3(128, 5e5, 8.0, 1.0, 4.0, 8192)
        tq_, tk = upload(b, qx), upload(b, kx)
        b.rope(tq_, tk, pos, 5e5, 128)
        outs.append((download(b, tq_), download(b, tk)))
        b.close()
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])
    with pytest.raises(ModelConfigError, match="rope frequencies from GGUF"):
        b = CudaBackend(0)
        try:
            b.precompute_rope_freqs_gguf(128, tmp_path / "missing.gguf")
        finally:
            b.close()


def test_embedding_through_backend(be):
    table = np.random.default_rng(2).standard_normal((256, 64)).astype(np.float32) * 0.02
    tt = upload(be, table, FB_BF16)
    out = be.alloc([33, 64], FB_BF16)
    ids = np.r_[np.arange(32), 999].astype(np.uint32)
    be.embedding(ids, tt, out)
    exp = ops.embedding(ops.round_to(table, "bf16"), ids)
    assert np.array_equal(download(be, out), exp)


def test_timers(be):
    t = be.create_timer()
    be.start_timer(t)
    ms = be.stop_timer(t)
    assert ms >= 0.0
    be.destroy_timer(t)
    with pytest.raises(BackendError):
        be.destroy_timer(t)


def test_turboquant_compress_trait_method(be):
    d, H, T, bits = 128, 8, 16, 4
    rng = np.random.default_rng(3)
    x = ops.round_to(rng.standard_normal((T, H, d)), "f16")
    pi = K.tq_rotation_matrix(d, 42)
    c, _ = K.tq_codebook(d, bits)
    tx = upload(be, x)
    tr = be.alloc([d, d], FB_FP32)
    be.copy_to_device(tr, pi)
    tc = be.alloc([16], FB_FP32)
    be.copy_to_device(tc, c)
    tp = be.alloc([T, H * 64], FB_INT8)
    tn = be.alloc([T, H], FB_FP16)
    be.turboquant_compress(tx, tr, tc, bits, tp, tn)
    pc, nc, _ = tq.compress_c(ops.to_storage_bytes(x, "f16").reshape(x.shape), tq.INPUT_F16, pi, c, bits)
    assert np.array_equal(be.copy_to_host(tp).reshape(T, -1), pc)
    assert np.array_equal(be.copy_to_host(tn).view(np.uint16).reshape(T, H), nc)
    bad = be.alloc([8], FB_FP32)
    with pytest.raises(InvalidShape, match="centroid table has 8 entries"):
        be.turboquant_compress(tx, tr, bad, bits, tp, tn)


# ── quantized paged KV cache ────────────────────────────────────────────────

def test_quantized_cache_append_matches_reference_placement(be):
    """Two sequences, uneven appends across 2 layers; pool bytes equal the CPU restatement
    of append_kv (compress to scratch, then place rows through the block table)."""
    H, d, L, NB = 8, 128, 2, 12
    cfg = TurboQuantConfig(key_bits=4, value_bits=3)
    cache = QuantizedKvCache(be, NB, L, H, d, cfg)
    ref = tq.QuantizedKvCache(NB, L, H, d, tq.TurboQuantConfig(key_bits=4, value_bits=3))
    a, b_ = cache.alloc(), cache.alloc()
    ra, rb = ref.alloc(), ref.alloc()
    rng = np.random.default_rng(9)
    for sid, rid, n in [(a, ra, 5), (b_, rb, 20), (a, ra, 13), (a, ra, 1), (b_, rb, 16)]:
        for layer in range(L):
            kx = ops.round_to(rng.standard_normal((n, H, d)), "f16")
            vx = ops.round_to(rng.standard_normal((n, H, d)), "f16")
            cache.append_kv(sid, layer, upload(be, kx), upload(be, vx))
            kb, vb = cfg.key_bits, cfg.value_bits
            kpi = tq.generate_rotation_matrix(d, tq.rotation_seeds(42, layer)[0])
            vpi = tq.generate_rotation_matrix(d, tq.rotation_seeds(42, layer)[1])
            kp, kn, _ = tq.compress_c(ops.to_storage_bytes(kx, "f16").reshape(kx.shape), tq.INPUT_F16, kpi,
                                      tq.get_codebook(d, kb).centroids, kb)
            vp, vn, _ = tq.compress_c(ops.to_storage_bytes(vx, "f16").reshape(vx.shape), tq.INPUT_F16, vpi,
                                      tq.get_codebook(d, vb).centroids, vb)
            ref.append_kv(rid, layer, kp, kn, vp, vn)
    assert cache.block_table(a) == ref.seqs[ra].block_table
    assert cache.block_table(b_) == ref.seqs[rb].block_table
    assert cache.seq_len(a) == 19 and cache.seq_len(b_) == 36
    be.synchronize()
    for layer in range(L):
        for kv in range(2):
            p = cache.pool(layer, kv)
            P = d * p["bits"] // 8
            rows = NB * 16
            # only rows that hold tokens are compared (the rest is never written)
            used = np.concatenate([ref.slots(s, 0, ref.seqs[s].current_len) for s in (ra, rb)])
            tp = be.register_external(p["packed"], [rows, H * P], FB_INT8)
            tn = be.register_external(p["norms"], [rows, H], FB_FP16)
            packed = be.copy_to_host(tp).reshape(rows, H * P)
            norms = be.copy_to_host(tn).view(np.uint16).reshape(rows, H)
            assert np.array_equal(packed[used], ref.pool_packed[layer][kv][used])
            assert np.array_equal(norms[used], ref.pool_norms[layer][kv][used])
    # dequant through the cache
    out = be.alloc([19, H, d], FB_FP32)
    cache.dequant(a, 1, 0, 19, out)
    got = download(be, out)
    assert np.all(np.isfinite(got))
    # errors and accounting
    with pytest.raises(KvCacheError, match="invalid handle: 77"):
        cache.append_kv(77, 0, upload(be, np.zeros((1, H, d))), upload(be, np.zeros((1, H, d))))
    free_before = cache.num_free_blocks()
    cache.free(a)
    assert cache.num_free_blocks() == free_before + len(ref.seqs[ra].block_table)
    with pytest.raises(KvCacheError):
        cache.free(a)
    cache.destroy()


def test_quantized_cache_attention_matches_statement(be):
    """Attention through the cache manager (batched.rs:143-193): a sequence grown by uneven appends
    over three layers (the first and last protected: 8-bit codes), then three query tokens at its end
    against the float64 statement of attention_paged_tq.cu on the cache's own pools."""
    H, d, L, NB, Hq = 8, 128, 3, 20, 32
    cfg = TurboQuantConfig(key_bits=4, value_bits=2, protected_bits=8, protected_layers=1)
    cache = QuantizedKvCache(be, NB, L, H, d, cfg)
    a = cache.alloc()
    rng = np.random.default_rng(12)
    for n in (37, 1, 90, 5):
        for layer in range(L):
            cache.append_kv(a, layer, upload(be, rng.standard_normal((n, H, d)) * 1.5),
                            upload(be, rng.standard_normal((n, H, d))))
    T = cache.seq_len(a)
    table = np.array(cache.block_table(a), np.int32)
    be.synchronize()
    for layer in range(L):
        q = ops.round_to(rng.standard_normal((3, Hq, d)), "f16")
        out = be.alloc([3, Hq, d], FB_FP16)
        cache.attention(a, layer, upload(be, q), T, T - 3, out)
        got = download(be, out)
        pools = []
        for kv in range(2):
            p = cache.pool(layer, kv)
            P = d * p["bits"] // 8
            rows = NB * 16
            tp = be.register_external(p["packed"], [rows, H * P], FB_INT8)
            tn = be.register_external(p["norms"], [rows, H], FB_FP16)
            tr = be.register_external(p["rotation"], [d, d], FB_FP32)
            tc = be.register_external(p["centroids"], [1 << p["bits"]], FB_FP32)
            pools.append((be.copy_to_host(tp).reshape(rows, H * P),
                          be.copy_to_host(tn).view(np.float16).astype(np.float64).reshape(rows, H),
                          be.copy_to_host(tr).view(np.float32).reshape(d, d),
                          be.copy_to_host(tc).view(np.float32), p["bits"]))
        (kp, kn, kr, kc, kb), (vp, vn, vr, vc, vb) = pools
        assert (kb, vb) == ((4, 2) if layer == 1 else (8, 8))
        ref = tq.attention_paged_tq(q, kp, kn, vp, vn, table, T, T - 3, kr, vr, kc, vc, kb, vb, H)
        ops.assert_close_fp(got, ref, rel=2e-3, min_cos=0.9999, label=f"layer {layer}", dtype="f16")
    with pytest.raises(KvCacheError, match="past the sequence length"):
        cache.attention(a, 0, upload(be, np.zeros((1, Hq, d))), T + 1, T, be.alloc([1, Hq, d], FB_FP16))
    cache.destroy()


def test_paged_cache_append_and_attention(be):
    """PagedKvCacheManager: uneven appends over two layers place rows through the block table
    (one block up front, new blocks on layer 0), the manager's attention meets the FP bar of
    attention_paged.cu's statement, and running out of blocks is OutOfMemory."""
    H, d, L, NB, Hq = 8, 128, 2, 12, 32
    cache = PagedKvCache(be, NB, L, H, d, FB_FP16)
    a = cache.alloc()
    assert cache.num_free_blocks() == NB - 1 and cache.block_table(a) != []
    rng = np.random.default_rng(13)
    keys = {l: [] for l in range(L)}
    vals = {l: [] for l in range(L)}
    for n in (10, 6, 1, 40):
        for layer in range(L):
            kx = ops.round_to(rng.standard_normal((n, H, d)), "f16")
            vx = ops.round_to(rng.standard_normal((n, H, d)), "f16")
            keys[layer].append(kx)
            vals[layer].append(vx)
            cache.append_kv(a, layer, upload(be, kx), upload(be, vx))
    T = cache.seq_len(a)
    assert T == 57 and cache.last_block_tokens(a) == 57 - 48
    table = np.array(cache.block_table(a), np.int32)
    assert len(table) == 4
    be.synchronize()
    pos = np.arange(T)
    rows = table[pos // 16] * 16 + pos % 16
    for layer in range(L):
        p = cache.pool(layer)
        tk = be.register_external(p["k"], [NB * 16, H, d], FB_FP16)
        tv = be.register_external(p["v"], [NB * 16, H, d], FB_FP16)
        kpool = be.copy_to_host(tk).view(np.float16).astype(np.float32).reshape(NB * 16, H, d)
        vpool = be.copy_to_host(tv).view(np.float16).astype(np.float32).reshape(NB * 16, H, d)
        assert np.array_equal(kpool[rows], np.concatenate(keys[layer]))
        assert np.array_equal(vpool[rows], np.concatenate(vals[layer]))
        q = ops.round_to(rng.standard_normal((2, Hq, d)), "f16")
        out = be.alloc([2, Hq, d], FB_FP16)
        cache.attention(a, layer, upload(be, q), T, T - 2, out)
        # the statement sees only the rows the sequence wrote (the other pool rows were never initialised)
        kused, vused = np.zeros_like(kpool), np.zeros_like(vpool)
        kused[rows], vused[rows] = kpool[rows], vpool[rows]
        ref = ops.attention_paged(q, kused, vused, table, T, T - 2)
        ops.assert_close_fp(download(be, out), ref, rel=2e-3, min_cos=0.9999, label=f"layer {layer}", dtype="f16")
    b_ = cache.alloc()
    with pytest.raises(OutOfMemory):
        for _ in range(20):
            for layer in range(L):
                cache.append_kv(b_, layer, upload(be, np.zeros((16, H, d))), upload(be, np.zeros((16, H, d))))
    free_before = cache.num_free_blocks()
    cache.free(a)
    assert cache.num_free_blocks() == free_before + len(table)
    with pytest.raises(KvCacheError, match="invalid handle"):
        cache.free(a)
    cache.destroy()


def test_quantized_cache_out_of_blocks(be):
    cache = QuantizedKvCache(be, 2, 1, 2, 16, TurboQuantConfig())
    h = cache.alloc()
    x = upload(be, np.ones((40, 2, 16)))
    with pytest.raises(OutOfMemory, match="out of device memory"):
        cache.append_kv(h, 0, x, x)
    cache.destroy()
