"""GPU parity of TurboQuant compress / dequantize against the exact CPU oracle.

Bar (north star): codebook indices and packed bytes bit-exact — every
coordinate, not just all but 1e-6 of them — and the fp16 norms bit-exact;
dequantized outputs within the FP tolerance of the float32 oracle (here they
are bit-exact in float32 output, since the dequant kernel evaluates the same
sequential sum). The pool placement (block table, start position) is
bit-exact by construction and checked byte for byte.
"""

import numpy as np
import pytest
import torch

from fracture_b200 import _lib
from fracture_b200 import kernels as K
from oracle import ops, turboquant as tq

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TDT = {"f16": torch.float16, "bf16": torch.bfloat16}
KIND = {"f16": tq.INPUT_F16, "bf16": tq.INPUT_BF16}


def make_input(T, H, d, dt, seed, outliers=0.005):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, H, d)).astype(np.float32)
    x[rng.random(x.shape) < outliers] *= 10.0
    x = ops.round_to(x, dt)
    return x, ops.to_storage_bytes(x, dt).reshape(x.shape)


def dev(x, dt):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(DEV).to(TDT[dt])


def tables(d, bits, seed):
    c, _ = K.tq_codebook(d, bits)
    return K.tq_rotation_matrix(d, seed), c


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("bits", [2, 3, 4, 8])
@pytest.mark.parametrize("T,H,d", [(64, 8, 128), (4, 2, 16), (7, 3, 32), (33, 8, 128), (5, 3, 33)])
def test_compress_bit_exact_compact_layout(dt, bits, T, H, d):
    x, raw = make_input(T, H, d, dt, seed=bits * 100 + T)
    pi, c = tables(d, bits, 42)
    P = tq.TurboQuantConfig.packed_dim_per_head(d, bits)
    packed = torch.zeros((T, H * P), dtype=torch.uint8, device=DEV)
    norms = torch.zeros((T, H), dtype=torch.float16, device=DEV)
    K.tq_compress_paged(dev(x, dt), torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV), bits, packed, norms)
    torch.cuda.synchronize()
    pc, nc, _ = tq.compress_c(raw, KIND[dt], pi, c, bits, num_threads=4)
    assert np.array_equal(packed.cpu().numpy(), pc)
    assert np.array_equal(norms.cpu().numpy().view(np.uint16), nc)


def test_reference_abi_compress_decompress_fp16():
    """launch_turboquant_compress / _decompress with the reference's argument lists."""
    from fracture_b200 import _lib

    lib = _lib.load()
    T, H, d, bits = 16, 8, 128, 4
    x, raw = make_input(T, H, d, "f16", 5)
    pi, c = tables(d, bits, 542)
    P = d * bits // 8
    tx = dev(x, "f16")
    tpi, tc = torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV)
    packed = torch.zeros((T, H * P), dtype=torch.uint8, device=DEV)
    norms = torch.zeros((T, H), dtype=torch.float16, device=DEV)
    s = torch.cuda.current_stream().cuda_stream
    assert lib.launch_turboquant_compress(tx.data_ptr(), tpi.data_ptr(), tc.data_ptr(), packed.data_ptr(),
                                          norms.data_ptr(), T, H, d, 16, bits, P, s) == 0
    out = torch.zeros((T, H, d), dtype=torch.float16, device=DEV)
    assert lib.launch_turboquant_decompress(packed.data_ptr(), norms.data_ptr(), tpi.data_ptr(), tc.data_ptr(),
                                            out.data_ptr(), T, H, d, bits, P, s) == 0
    torch.cuda.synchronize()
    pc, nc, _ = tq.compress_c(raw, tq.INPUT_F16, pi, c, bits)
    assert np.array_equal(packed.cpu().numpy(), pc)
    ref = tq.decompress_c(pc, nc, pi, c, bits, H, d)
    ops.assert_close_fp(out.float().cpu().numpy(), ref, label="decompress fp16")


@pytest.mark.parametrize("bits", [3, 4])
@pytest.mark.parametrize("start_pos", [0, 5, 16])
def test_compress_into_paged_pool(bits, start_pos):
    """Random block table, unaligned start: every token lands in block_table[pos/16]*16 + pos%16."""
    T, H, d, nblocks = 70, 8, 128, 40
    x, raw = make_input(T, H, d, "f16", 11 + bits)
    pi, c = tables(d, bits, 1042)
    rng = np.random.default_rng(3)
    table = rng.permutation(nblocks).astype(np.int32)
    P = d * bits // 8
    rows = nblocks * 16
    packed = torch.full((rows, H * P), 0xAB, dtype=torch.uint8, device=DEV)
    norms = torch.full((rows, H), 0x5555, dtype=torch.int16, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    K.tq_compress_paged(dev(x, "f16"), torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV), bits, packed,
                        norms, block_table=torch.from_numpy(table).to(DEV), start_pos=start_pos, err=err)
    torch.cuda.synchronize()
    assert err.item() == 0
    pc, nc, _ = tq.compress_c(raw, tq.INPUT_F16, pi, c, bits)
    exp_p = np.full((rows, H * P), 0xAB, np.uint8)
    exp_n = np.full((rows, H), 0x5555, np.uint16)
    pos = start_pos + np.arange(T)
    slots = table[pos // 16] * 16 + pos % 16
    exp_p[slots] = pc
    exp_n[slots] = nc
    assert np.array_equal(packed.cpu().numpy(), exp_p)
    assert np.array_equal(norms.cpu().numpy().view(np.uint16), exp_n)
    # dequantize back out of the pool
    out = torch.zeros((T, H, d), dtype=torch.float32, device=DEV)
    K.tq_dequant_paged(packed, norms, torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV), bits, out,
                       block_table=torch.from_numpy(table).to(DEV), start_pos=start_pos)
    torch.cuda.synchronize()
    ref = tq.decompress_c(pc, nc, pi, c, bits, H, d)
    assert np.array_equal(out.cpu().numpy(), ref)


def test_out_of_range_slots_are_skipped_and_counted():
    T, H, d, bits = 20, 2, 16, 4
    x, _ = make_input(T, H, d, "f16", 1)
    pi, c = tables(d, bits, 42)
    table = np.array([0, -1], dtype=np.int32)  # second block missing
    packed = torch.zeros((16, H * 8), dtype=torch.uint8, device=DEV)
    norms = torch.zeros((16, H), dtype=torch.float16, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    K.tq_compress_paged(dev(x, "f16"), torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV), bits, packed,
                        norms, block_table=torch.from_numpy(table).to(DEV), err=err)
    torch.cuda.synchronize()
    assert err.item() > 0  # tokens 16..19 have no block; nothing was written for them
    assert packed.cpu().numpy().any()


# ── small calls (decode steps): the few-vectors-per-CTA exact kernels ──

@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("T,H,d,bits", [(1, 8, 128, 4), (37, 8, 128, 4), (77, 8, 128, 3), (125, 8, 128, 2),
                                        (9, 3, 64, 8), (5, 3, 33, 4), (40, 2, 192, 4)])
def test_small_call_compress_bit_exact(dt, T, H, d, bits):
    """Calls of up to 1024 head vectors (1, 2 or 4 vectors per CTA, the last CTA partial) into a
    paged pool with an unaligned start and one missing block: pool bytes and norms bit-exact
    against the oracle, tokens of the missing block untouched and counted once per vector."""
    start = 3
    x, raw = make_input(T, H, d, "f16" if dt == "f32" else dt, 900 + T * H + d)
    if dt == "f32":
        x = x.astype(np.float32) * np.float32(1.0 + 2.0 ** -13)  # values off the fp16 grid
        raw = x
    pi, c = tables(d, bits, 5 + d)
    P = (d * bits + 7) // 8
    nblk = (start + T + 15) // 16 + 2
    table = np.random.default_rng(T).permutation(nblk).astype(np.int32)
    missing = (start + T - 1) // 16 if T > 20 else -1
    if missing >= 0:
        table[missing] = -1
    rows = nblk * 16
    packed = torch.full((rows, H * P), 0xAB, dtype=torch.uint8, device=DEV)
    norms = torch.full((rows, H), 0x5555, dtype=torch.int16, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    xin = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(DEV)
    if dt != "f32":
        xin = xin.to(TDT[dt])
    K.tq_compress_paged(xin, torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV), bits, packed, norms,
                        block_table=torch.from_numpy(table).to(DEV), start_pos=start, err=err)
    torch.cuda.synchronize()
    kind = {"f16": tq.INPUT_F16, "bf16": tq.INPUT_BF16, "f32": tq.INPUT_F32}[dt]
    pc, nc, _ = tq.compress_c(raw, kind, pi, c, bits)
    pos = start + np.arange(T)
    have = table[pos // 16] >= 0
    slots = table[pos // 16] * 16 + pos % 16
    exp_p = np.full((rows, H * P), 0xAB, np.uint8)
    exp_n = np.full((rows, H), 0x5555, np.uint16)
    exp_p[slots[have]] = pc[have]
    exp_n[slots[have]] = nc[have]
    assert np.array_equal(packed.cpu().numpy(), exp_p)
    assert np.array_equal(norms.cpu().numpy().view(np.uint16), exp_n)
    assert err.item() == int((~have).sum()) * H


@pytest.mark.parametrize("entry", ["paged", "slots"])
@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("T,H,d,kb,vb", [(1, 8, 128, 4, 2), (32, 8, 128, 4, 4), (128, 8, 128, 4, 2),
                                         (77, 8, 128, 3, 3), (9, 3, 64, 8, 2), (5, 3, 33, 2, 4)])
def test_small_call_compress_kv_one_launch(entry, dt, T, H, d, kb, vb):
    """K and V of a decode-sized append in one small-call launch (its CTAs split between K and V,
    the vectors per CTA chosen from both calls' vectors; 128 x 8 is 1024 vectors each, the
    small-call limit), through the block-table entry point (unaligned start) and the slot-map one
    (one token without a pool row): pool bytes and norms bit-exact against the oracle, rows not
    written left as they were, the skipped token counted once per head vector of K and of V, and
    one launch counted for the pair."""
    xk, rk = make_input(T, H, d, dt, seed=1300 + T * H + d)
    xv, rv = make_input(T, H, d, dt, seed=1301 + T * H + d)
    pik, ck = tables(d, kb, 42)
    piv, cv = tables(d, vb, 542)
    rng = np.random.default_rng(T + d)
    start = 3
    nblk = (start + T + 15) // 16 + 2
    rows = nblk * 16
    if entry == "paged":
        table = rng.permutation(nblk).astype(np.int32)
        pos = start + np.arange(T)
        slots = (table[pos // 16] * 16 + pos % 16).astype(np.int64)
    else:
        slots = rng.permutation(rows)[:T].astype(np.int64)
        if T > 4:
            slots[T // 2] = -1
    have = slots >= 0
    pools = []
    for b in (kb, vb):
        P = (d * b + 7) // 8
        pools.append((torch.full((rows, H * P), 0xAB, dtype=torch.uint8, device=DEV),
                      torch.full((rows, H), 0x5555, dtype=torch.int16, device=DEV)))
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    args = (dev(xk, dt), dev(xv, dt), torch.from_numpy(pik).to(DEV), torch.from_numpy(piv).to(DEV),
            torch.from_numpy(ck).to(DEV), torch.from_numpy(cv).to(DEV), kb, vb, pools[0][0], pools[0][1],
            pools[1][0], pools[1][1])
    before = K.tq_path_counts()
    if entry == "paged":
        K.tq_compress_kv_paged(*args, block_table=torch.from_numpy(table).to(DEV), start_pos=start, err=err)
    else:
        K.tq_compress_kv_slots(*args, torch.from_numpy(slots).to(DEV), err=err)
    torch.cuda.synchronize()
    after = K.tq_path_counts()
    assert after["compress_kv_small"] - before["compress_kv_small"] == 1, (before, after)
    assert after["compress_small"] == before["compress_small"], (before, after)
    assert err.item() == int((~have).sum()) * H * 2
    for (packed, norms), raw, pi, c, b in ((pools[0], rk, pik, ck, kb), (pools[1], rv, piv, cv, vb)):
        pc, nc, _ = tq.compress_c(raw, KIND[dt], pi, c, b)
        exp_p = np.full((rows, H * ((d * b + 7) // 8)), 0xAB, np.uint8)
        exp_n = np.full((rows, H), 0x5555, np.uint16)
        exp_p[slots[have]] = pc[have]
        exp_n[slots[have]] = nc[have]
        assert np.array_equal(packed.cpu().numpy(), exp_p), f"{b}-bit codes"
        assert np.array_equal(norms.cpu().numpy().view(np.uint16), exp_n), f"{b}-bit norms"


@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("T,H,d,bits", [(1, 8, 128, 4), (24, 8, 128, 4), (19, 3, 64, 3), (7, 3, 33, 2)])
def test_small_call_dequant_bit_exact(dt, T, H, d, bits):
    """Calls of up to 192 head vectors take the exact small-call kernel: the float32 statement,
    rounded once to the output type; a token whose block is missing gives zeros."""
    start = 5
    x, raw = make_input(T, H, d, "f16", 300 + T + d)
    pi, c = tables(d, bits, 77)
    P = (d * bits + 7) // 8
    nblk = (start + T + 15) // 16
    table = np.random.default_rng(d).permutation(nblk).astype(np.int32)
    rows = nblk * 16
    tt = torch.from_numpy(table).to(DEV)
    tpi, tc = torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV)
    packed = torch.zeros((rows, H * P), dtype=torch.uint8, device=DEV)
    norms = torch.zeros((rows, H), dtype=torch.float16, device=DEV)
    K.tq_compress_paged(dev(x, "f16"), tpi, tc, bits, packed, norms, block_table=tt, start_pos=start)
    if T > 4:
        tt[(start + T - 1) // 16] = -1
    odt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[dt]
    out = torch.full((T, H, d), 7.0, dtype=odt, device=DEV)
    K.tq_dequant_paged(packed, norms, tpi, tc, bits, out, block_table=tt, start_pos=start)
    torch.cuda.synchronize()
    pc, nc, _ = tq.compress_c(raw, tq.INPUT_F16, pi, c, bits)
    ref = tq.decompress_c(pc, nc, pi, c, bits, H, d).reshape(T, H, d)
    if T > 4:
        pos = start + np.arange(T)
        ref[pos // 16 == (start + T - 1) // 16] = 0.0
    exp = torch.from_numpy(ref).to(odt).float().numpy()
    assert np.array_equal(out.float().cpu().numpy(), exp)


@pytest.mark.parametrize("bits,min_cos", [(4, 0.95), (2, 0.80), (8, 0.999)])
def test_reference_gpu_roundtrip_thresholds(bits, min_cos):
    """turboquant_gpu.rs:87-430: head_dim 16, 2 heads, 4 tokens, rotation-matrix entries as data."""
    d, H, T = 16, 2, 4
    numel = T * H * d
    side = max(int(np.ceil(np.sqrt(numel))), 2)
    x = K.tq_rotation_matrix(side, 12345).ravel()[:numel].astype(np.float16).astype(np.float32).reshape(T, H, d)
    pi, c = tables(d, bits, 42)
    P = tq.TurboQuantConfig.packed_dim_per_head(d, bits)
    packed = torch.zeros((T, H * P), dtype=torch.uint8, device=DEV)
    norms = torch.zeros((T, H), dtype=torch.float16, device=DEV)
    tpi, tc = torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV)
    K.tq_compress_paged(dev(x, "f16"), tpi, tc, bits, packed, norms)
    out = torch.zeros((T, H, d), dtype=torch.float16, device=DEV)
    K.tq_dequant_paged(packed, norms, tpi, tc, bits, out)
    torch.cuda.synchronize()
    o = out.float().cpu().numpy()
    n = norms.float().cpu().numpy()
    for t in range(T):
        for h in range(H):
            a, b = x[t, h], o[t, h]
            assert a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-10) > min_cos
            assert abs(n[t, h] - np.linalg.norm(a)) / np.linalg.norm(a) < 0.02


def test_zero_vectors():
    T, H, d, bits = 3, 8, 128, 4
    x = np.zeros((T, H, d), np.float32)
    pi, c = tables(d, bits, 42)
    packed = torch.zeros((T, H * 64), dtype=torch.uint8, device=DEV)
    norms = torch.ones((T, H), dtype=torch.float16, device=DEV)
    K.tq_compress_paged(dev(x, "f16"), torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV), bits, packed, norms)
    out = torch.ones((T, H, d), dtype=torch.float16, device=DEV)
    K.tq_dequant_paged(packed, norms, torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV), bits, out)
    torch.cuda.synchronize()
    assert not norms.float().cpu().numpy().any()
    assert np.all(np.isfinite(out.float().cpu().numpy())) and np.abs(out.float().cpu().numpy()).max() < 1e-6
    pc, nc, _ = tq.compress_c(np.zeros((T, H, d), np.uint16), tq.INPUT_F16, pi, c, bits)
    assert np.array_equal(packed.cpu().numpy(), pc)


@pytest.mark.parametrize("bits", [3, 4])
def test_config4_scale_bit_exact_sample(bits):
    """BASELINE config 4 shape (65536 x 8 x 128, 0.5% outliers x10) on the GPU; the C oracle
    checks a 4096-token sample bit for bit, and the pool round trip is checked everywhere."""
    T, H, d = 65536, 8, 128
    g = torch.Generator(device=DEV).manual_seed(4)
    x = torch.randn((T, H, d), generator=g, device=DEV)
    x = torch.where(torch.rand((T, H, d), generator=g, device=DEV) < 0.005, x * 10.0, x).to(torch.float16)
    pi, c = tables(d, bits, 42)
    tpi, tc = torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV)
    P = d * bits // 8
    packed = torch.zeros((T, H * P), dtype=torch.uint8, device=DEV)
    norms = torch.zeros((T, H), dtype=torch.float16, device=DEV)
    K.tq_compress_paged(x, tpi, tc, bits, packed, norms)
    torch.cuda.synchronize()
    sl = slice(T - 4096, T)
    raw = x[sl].cpu().numpy().view(np.uint16)
    pc, nc, _ = tq.compress_c(raw, tq.INPUT_F16, pi, c, bits, num_threads=8)
    assert np.array_equal(packed[sl].cpu().numpy(), pc)
    assert np.array_equal(norms[sl].cpu().numpy().view(np.uint16), nc)
    out = torch.empty((T, H, d), dtype=torch.float16, device=DEV)
    K.tq_dequant_paged(packed, norms, tpi, tc, bits, out)
    torch.cuda.synchronize()
    xf, of = x.float(), out.float()
    cos = (xf * of).sum(-1) / (xf.norm(dim=-1) * of.norm(dim=-1) + 1e-10)
    assert cos.min().item() > (0.95 if bits == 4 else 0.90)  # turboquant_gpu.rs: >0.95 at 4 bits


# ── tensor-core path (head_dim 128, 2/3/4 bits, FP16/BF16): full-size bit-exactness ──

@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("bits", [2, 3, 4])
def test_tensor_core_path_bit_exact_many_tiles(dt, bits):
    """8219 tokens x 8 heads = 513+ tiles (last one partial), every vector checked against
    the exact C statement; the kernel must not have timed out."""
    from fracture_b200 import _lib

    T, H, d = 8219, 8, 128
    x, raw = make_input(T, H, d, dt, seed=77 + bits)
    pi, c = tables(d, bits, 5042)
    P = d * bits // 8
    packed = torch.zeros((T, H * P), dtype=torch.uint8, device=DEV)
    norms = torch.zeros((T, H), dtype=torch.float16, device=DEV)
    before = _lib.load().fb_tq_timeouts()
    K.tq_compress_paged(dev(x, dt), torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV), bits, packed, norms)
    torch.cuda.synchronize()
    assert _lib.load().fb_tq_timeouts() == before
    pc, nc, _ = tq.compress_c(raw, KIND[dt], pi, c, bits, num_threads=8)
    got_p, got_n = packed.cpu().numpy(), norms.cpu().numpy().view(np.uint16)
    bad_rows = np.nonzero(np.any(got_p != pc, axis=1) | np.any(got_n != nc, axis=1))[0]
    assert bad_rows.size == 0, f"{bad_rows.size} token rows differ, first {bad_rows[:5]}"


SMALL_CALL_VECTORS = 1024  # kTqSmallCompressVectors: larger calls take the tensor-core kernel


def _compress_on_path(x, dt, pi, c, bits, expect_tensor_core):
    """Compresses x ([T, H, 128], values) and checks which kernel family served the call."""
    T, H, d = x.shape
    P = d * bits // 8
    packed = torch.zeros((T, H * P), dtype=torch.uint8, device=DEV)
    norms = torch.zeros((T, H), dtype=torch.float16, device=DEV)
    before = K.tq_path_counts()
    K.tq_compress_paged(dev(x, dt), torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV), bits, packed, norms)
    torch.cuda.synchronize()
    after = K.tq_path_counts()
    path = "compress_tensor_core" if expect_tensor_core else "compress_small"
    assert after[path] == before[path] + 1, (before, after)
    return packed.cpu().numpy(), norms.cpu().numpy()


@pytest.mark.parametrize("T", [40, 300])
def test_tensor_core_path_adversarial_vectors(T):
    """Vectors aligned with rows of Pi (|y_i| = 1), zero vectors, tiny and huge fp16 values,
    and vectors placed exactly on decision boundaries, at the start and in the middle of the
    call: 40 tokens x 8 heads take the small-call kernel, 300 x 8 (2400 vectors) the tensor-core
    kernel (the call asserts which one ran). Bit-exact against the exact statement."""
    H, d, bits = 8, 128, 4
    pi, c = tables(d, bits, 42)
    rng = np.random.default_rng(5)
    x = rng.standard_normal((T, H, d)).astype(np.float32)
    mids = (c[:-1] + c[1:]) / 2
    for r0 in sorted({0, T // 2 + 3}):
        x[r0 + 0, :] = pi[:H, :]       # x = row i of Pi  ->  y = e_i
        x[r0 + 1, :] = 0.0
        x[r0 + 2, :] = 6e-8            # fp16 subnormal
        x[r0 + 3, :] = 60000.0
        x[r0 + 4, :, :] = 0.0
        x[r0 + 4, :, 0] = 1.0          # y = Pi[:, 0]
        for h in range(H):             # y lands on a boundary (to fp16 rounding of x)
            y = rng.choice(mids, d)
            x[r0 + 5, h] = pi.T.astype(np.float64) @ y
    x = ops.round_to(x, "f16")
    raw = ops.to_storage_bytes(x, "f16").reshape(x.shape)
    got_p, got_n = _compress_on_path(x, "f16", pi, c, bits, T * H > SMALL_CALL_VECTORS)
    pc, nc, _ = tq.compress_c(raw, tq.INPUT_F16, pi, c, bits, num_threads=4)
    assert np.array_equal(got_p, pc)
    assert np.array_equal(got_n.view(np.uint16), nc)


def _boundary_codebook(values, n_levels):
    """Centroids whose decision boundaries (c_k + c_{k+1}) / 2 sit on chosen y values.

    Walks upwards from c_0 (just below the smallest value): the next boundary is the smallest
    of ``values`` between 0.012 and 0.03 above the current centroid (else a synthetic one 0.015 above), and the next
    centroid mirrors the current one across it, so centroids increase by at least 0.024
    and boundaries are at least 0.024 apart."""
    vals = np.sort(np.asarray(values, np.float64))
    c = [max(-0.42, float(vals[0]) - 0.013)]
    mids = []
    while len(c) < n_levels:
        lo, hi = c[-1] + 0.012, c[-1] + 0.03
        pick = vals[(vals > lo) & (vals <= hi)]
        if mids:
            pick = pick[pick - mids[-1] >= 0.025]
        v = float(pick[0]) if pick.size else c[-1] + 0.015
        mids.append(v)
        c.append(2.0 * v - c[-1])
    return np.array(c, dtype=np.float32), np.array(mids)


def test_tensor_core_path_queue_overflow():
    """Every row has 15 coordinates on a decision boundary, so the exact-settle queue overflows:
    rows beyond its capacity are settled inside the main kernel, and the partly reserved
    entries are voided. The result still equals the exact statement bit for bit."""
    T, H, d, bits = 300, 8, 128, 4
    pi = K.tq_rotation_matrix(d, 42)
    rng = np.random.default_rng(11)
    c, m = _boundary_codebook(pi[:, 0], 1 << bits)
    assert np.all(np.diff(c) > 0)
    # x = v * e_0 with v + 1e-8 == v in float32: x / (norm + 1e-8) = e_0 and y = Pi[:, 0] exactly
    x = np.zeros((T, H, d), np.float32)
    x[:, :, 0] = rng.choice([0.5, 1.0, 3.0, 100.0, -2.0], size=(T, H))
    raw = ops.to_storage_bytes(x, "f16").reshape(x.shape)
    y = pi[:, 0]
    assert np.sum(np.min(np.abs(y[:, None] - m[None, :]), axis=1) < 1e-6) >= 10
    packed = torch.zeros((T, H * 64), dtype=torch.uint8, device=DEV)
    norms = torch.zeros((T, H), dtype=torch.float16, device=DEV)
    K.tq_compress_paged(dev(x, "f16"), torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV), bits, packed, norms)
    torch.cuda.synchronize()
    pc, nc, _ = tq.compress_c(raw, tq.INPUT_F16, pi, c, bits)
    assert np.array_equal(packed.cpu().numpy(), pc)
    assert np.array_equal(norms.cpu().numpy().view(np.uint16), nc)


@pytest.mark.parametrize("T", [64, 260])
@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_tensor_core_path_non_finite_rows(dt, T):
    """Rows holding NaN or +-inf (and, for BF16, values whose squares overflow float32) next to
    ordinary rows of the same warp, at the start and in the middle of the call: 64 x 8 vectors
    take the small-call kernel, 260 x 8 the tensor-core kernel (asserted), which keeps every table
    index in range. Every row equals the exact statement (NaN rows code to index 0; NaN norms
    compared as NaN)."""
    H, d, bits = 8, 128, 4
    x, _ = make_input(T, H, d, dt, seed=21)
    for r0 in sorted({0, T // 2 + 1}):
        x[r0 + 0, 1, 5] = np.nan
        x[r0 + 1, 2, 0] = np.inf
        x[r0 + 2, 3, 7] = -np.inf
        x[r0 + 3, 4, 9], x[r0 + 3, 4, 10] = np.inf, -np.inf
        x[r0 + 9, 0, :] = np.nan
        if dt == "bf16":
            x[r0 + 5, 6, :] = 1e30  # |x|^2 overflows float32: norm = inf, y = 0
            x[r0 + 6, 7, 3] = -3e38
    x = ops.round_to(x, dt)
    raw = ops.to_storage_bytes(x, dt).reshape(x.shape)
    pi, c = tables(d, bits, 42)
    got_p, got = _compress_on_path(x, dt, pi, c, bits, T * H > SMALL_CALL_VECTORS)
    pc, nc, _ = tq.compress_c(raw, KIND[dt], pi, c, bits, num_threads=4)
    assert np.array_equal(got_p, pc)
    exp = nc.view(np.float16)
    both_nan = np.isnan(got) & np.isnan(exp)
    assert np.array_equal(got.view(np.uint16)[~both_nan], nc[~both_nan])
    assert np.array_equal(np.isnan(got), np.isnan(exp))


@pytest.mark.parametrize("dt,kb,vb,T", [("f16", 4, 4, 4099), ("bf16", 4, 4, 1500), ("f16", 3, 3, 2053),
                                         ("f16", 2, 2, 300), ("f16", 4, 2, 3001), ("bf16", 4, 2, 1200),
                                         ("f16", 2, 4, 700), ("f16", 4, 4, 130), ("bf16", 3, 3, 20000)])
def test_compress_kv_one_launch_equals_the_statement(dt, kb, vb, T):
    """fb_launch_tq_compress_kv_paged: K and V of one append (shuffled block table, unaligned start)
    in one tensor-core launch whose grid is split between them (or two calls where the widths have
    no fused kernel, 2/4, or the call is small). Every packed byte and norm equals the exact
    statement; the path counter shows which way it went. 20000 x 8 vectors (1250 tiles per job)
    splits the SMs in proportion; 130 x 8 (9 tiles) gives each job fewer CTAs than SMs."""
    H, d, start = 8, 128, 5
    xk, rk = make_input(T, H, d, dt, seed=900 + T)
    xv, rv = make_input(T, H, d, dt, seed=901 + T)
    pik, ck = tables(d, kb, 42)
    piv, cv = tables(d, vb, 542)
    nblk = (start + T + 15) // 16
    table = np.random.default_rng(T).permutation(nblk + 2)[:nblk].astype(np.int32)
    rows = (nblk + 2) * 16
    pools = [(torch.full((rows, H * d * b // 8), 0x5A, dtype=torch.uint8, device=DEV),
              torch.zeros((rows, H), dtype=torch.float16, device=DEV)) for b in (kb, vb)]
    before = K.tq_path_counts()
    K.tq_compress_kv_paged(dev(xk, dt), dev(xv, dt), torch.from_numpy(pik).to(DEV), torch.from_numpy(piv).to(DEV),
                           torch.from_numpy(ck).to(DEV), torch.from_numpy(cv).to(DEV), kb, vb, pools[0][0],
                           pools[0][1], pools[1][0], pools[1][1], block_table=torch.from_numpy(table).to(DEV),
                           start_pos=start)
    torch.cuda.synchronize()
    after = K.tq_path_counts()
    fused = T * H > SMALL_CALL_VECTORS and (kb == vb or (kb, vb) == (4, 2))
    assert after["compress_kv_fused"] - before["compress_kv_fused"] == (1 if fused else 0), (before, after)
    pos = start + np.arange(T)
    prow = table[pos // 16] * 16 + pos % 16
    for (packed, norms), raw, pi, c, b in ((pools[0], rk, pik, ck, kb), (pools[1], rv, piv, cv, vb)):
        pc, nc, _ = tq.compress_c(raw, KIND[dt], pi, c, b, num_threads=8)
        got_p, got_n = packed.cpu().numpy()[prow], norms.cpu().numpy().view(np.uint16)[prow]
        bad = np.nonzero(np.any(got_p != pc, axis=1) | np.any(got_n != nc, axis=1))[0]
        assert bad.size == 0, f"{b}-bit: {bad.size} token rows differ, first {bad[:5]}"


# ── tensor-core dequantize (head_dim 128, 2/3/4 bits, FP16/BF16 output) ──

@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("bits", [2, 3, 4])
def test_tensor_core_dequant_paged_many_tiles(dt, bits):
    """4099 tokens x 8 heads (257 tiles, the last one partial) from a shuffled paged pool with an
    unaligned start; against the float32 statement: within 3e-4 of the magnitude beyond the output
    dtype's rounding (the north-star bar is 2e-3) and cosine >= 0.9999."""
    T, H, d, start = 4099, 8, 128, 21
    x, raw = make_input(T, H, d, "f16", seed=300 + bits)
    pi, c = tables(d, bits, 4242)
    P = d * bits // 8
    nblk = (start + T + 15) // 16 + 3
    table = np.random.default_rng(bits).permutation(nblk).astype(np.int32)
    rows = nblk * 16
    tpi, tc, tt = torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV), torch.from_numpy(table).to(DEV)
    packed = torch.zeros((rows, H * P), dtype=torch.uint8, device=DEV)
    norms = torch.zeros((rows, H), dtype=torch.float16, device=DEV)
    K.tq_compress_paged(dev(x, "f16"), tpi, tc, bits, packed, norms, block_table=tt, start_pos=start)
    out = torch.full((T, H, d), 7.0, dtype=TDT[dt], device=DEV)
    before = _lib.load().fb_tq_timeouts()
    K.tq_dequant_paged(packed, norms, tpi, tc, bits, out, block_table=tt, start_pos=start)
    torch.cuda.synchronize()
    assert _lib.load().fb_tq_timeouts() == before
    pc, nc, _ = tq.compress_c(raw, tq.INPUT_F16, pi, c, bits, num_threads=8)
    ref = tq.decompress_c(pc, nc, pi, c, bits, H, d).reshape(T, H, d)
    got = out.float().cpu().numpy()
    ops.assert_close_fp(got, ref, rel=3e-4, min_cos=0.9999, label=f"tensor-core dequant {dt}/{bits}", dtype=dt)
    # every vector on its own
    num = (got * ref).sum(-1)
    den = np.linalg.norm(got, axis=-1) * np.linalg.norm(ref, axis=-1) + 1e-30
    assert (num / den).min() > 0.9999


@pytest.mark.parametrize("dt,kb,vb,T,H,start", [("f16", 4, 4, 4099, 8, 21), ("bf16", 4, 2, 2000, 8, 0),
                                               ("f16", 3, 3, 1500, 16, 5), ("f16", 2, 2, 700, 32, 13),
                                               ("bf16", 4, 4, 300, 64, 3), ("f16", 2, 4, 900, 8, 7)])
def test_dequant_kv_one_launch_with_missing_blocks(dt, kb, vb, T, H, start):
    """fb_launch_tq_dequant_kv_paged: K and V from shuffled pools in one launch (widths with a fused
    kernel; 2/4 goes as two calls), with two block-table entries negative and the pool ending 5 rows
    into the last block, so whole tiles, parts of tiles and parts of blocks have no pool row. Every
    token with a row equals the float32 statement (3e-4 of magnitude beyond the output rounding,
    cosine 0.9999 per vector); tokens without one are zero; the fused call equals the two separate
    calls bit for bit."""
    d = 128
    nblk = (start + T + 15) // 16
    table = np.random.default_rng(T + H).permutation(nblk).astype(np.int32)
    table[nblk // 3] = -1
    table[(2 * nblk) // 3] = -7
    rows = int(table.max()) * 16 + 5  # the highest block keeps only its first 5 rows
    tt = torch.from_numpy(table).to(DEV)
    pos = start + np.arange(T)
    slot = table[pos // 16].astype(np.int64) * 16 + pos % 16
    has_row = (table[pos // 16] >= 0) & (slot < rows)
    assert has_row.sum() < T and has_row.sum() > T // 2
    jobs = []
    for j, b in enumerate((kb, vb)):
        x, raw = make_input(T, H, d, "f16", seed=60 + 7 * j + T)
        pi, c = tables(d, b, 31 + j)
        P = d * b // 8
        packed = torch.zeros((rows, H * P), dtype=torch.uint8, device=DEV)
        norms = torch.zeros((rows, H), dtype=torch.float16, device=DEV)
        tpi, tc = torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV)
        # write only the tokens that have a row (the others would be refused and counted)
        err = torch.zeros(1, dtype=torch.int32, device=DEV)
        K.tq_compress_paged(dev(x, "f16"), tpi, tc, b, packed, norms, block_table=tt, start_pos=start, err=err)
        torch.cuda.synchronize()
        assert err.item() == (T - has_row.sum()) * H
        jobs.append(dict(x=x, raw=raw, pi=pi, c=c, b=b, packed=packed, norms=norms, tpi=tpi, tc=tc))
    outs = [torch.full((T, H, d), 7.0, dtype=TDT[dt], device=DEV) for _ in range(2)]
    before = K.tq_path_counts()
    K.tq_dequant_kv_paged(jobs[0]["packed"], jobs[0]["norms"], jobs[1]["packed"], jobs[1]["norms"], jobs[0]["tpi"],
                          jobs[1]["tpi"], jobs[0]["tc"], jobs[1]["tc"], kb, vb, outs[0], outs[1], block_table=tt,
                          start_pos=start)
    torch.cuda.synchronize()
    after = K.tq_path_counts()
    fused = kb == vb or (kb, vb) == (4, 2)
    assert after["dequant_kv_fused"] - before["dequant_kv_fused"] == (1 if fused else 0), (before, after)
    for j, jb in enumerate(jobs):
        sep = torch.full((T, H, d), 7.0, dtype=TDT[dt], device=DEV)
        K.tq_dequant_paged(jb["packed"], jb["norms"], jb["tpi"], jb["tc"], jb["b"], sep, block_table=tt,
                           start_pos=start)
        torch.cuda.synchronize()
        assert torch.equal(sep.view(torch.int16), outs[j].view(torch.int16)), f"job {j}: fused differs from separate"
        got = outs[j].float().cpu().numpy()
        assert not np.any(got[~has_row]), f"job {j}: a token without a pool row is not zero"
        pc, nc, _ = tq.compress_c(jb["raw"][has_row], tq.INPUT_F16, jb["pi"], jb["c"], jb["b"], num_threads=8)
        ref = tq.decompress_c(pc, nc, jb["pi"], jb["c"], jb["b"], H, d).reshape(-1, H, d)
        g = got[has_row]
        ops.assert_close_fp(g, ref, rel=3e-4, min_cos=0.9999, label=f"job {j} {dt}/{jb['b']}", dtype=dt)
        cos = (g * ref).sum(-1) / (np.linalg.norm(g, axis=-1) * np.linalg.norm(ref, axis=-1) + 1e-30)
        assert cos.min() > 0.9999


@pytest.mark.parametrize("H", [1, 3, 5, 7])
def test_tensor_core_dequant_odd_head_counts(H):
    """Token and head of each vector come from a division by the head count done by
    multiply-high and shifts; head counts that are not powers of two, over several waves of
    tiles, against the float32 statement."""
    T, d, bits, start = 160 * 128 // H + 7, 128, 4, 9
    x, raw = make_input(T, H, d, "f16", seed=40 + H)
    pi, c = tables(d, bits, 77)
    P = d * bits // 8
    nblk = (start + T + 15) // 16
    table = np.random.default_rng(H).permutation(nblk).astype(np.int32)
    tpi, tc, tt = torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV), torch.from_numpy(table).to(DEV)
    packed = torch.zeros((nblk * 16, H * P), dtype=torch.uint8, device=DEV)
    norms = torch.zeros((nblk * 16, H), dtype=torch.float16, device=DEV)
    K.tq_compress_paged(dev(x, "f16"), tpi, tc, bits, packed, norms, block_table=tt, start_pos=start)
    out = torch.full((T, H, d), 7.0, dtype=torch.float16, device=DEV)
    K.tq_dequant_paged(packed, norms, tpi, tc, bits, out, block_table=tt, start_pos=start)
    torch.cuda.synchronize()
    pc, nc, _ = tq.compress_c(raw, tq.INPUT_F16, pi, c, bits, num_threads=8)
    ref = tq.decompress_c(pc, nc, pi, c, bits, H, d).reshape(T, H, d)
    ops.assert_close_fp(out.float().cpu().numpy(), ref, rel=3e-4, min_cos=0.9999,
                        label=f"tensor-core dequant H={H}", dtype="f16")


def test_tensor_core_dequant_missing_blocks_give_zeros():
    """Tokens whose block-table entry is -1 dequantize to zeros, like the CUDA-core kernel."""
    T, H, d, bits = 300, 8, 128, 4
    x, _ = make_input(T, H, d, "f16", seed=5)
    pi, c = tables(d, bits, 42)
    nblk = (T + 15) // 16
    table = np.arange(nblk, dtype=np.int32)
    tpi, tc = torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV)
    packed = torch.zeros((nblk * 16, H * 64), dtype=torch.uint8, device=DEV)
    norms = torch.zeros((nblk * 16, H), dtype=torch.float16, device=DEV)
    K.tq_compress_paged(dev(x, "f16"), tpi, tc, bits, packed, norms, block_table=torch.from_numpy(table).to(DEV))
    table[[3, 7]] = -1
    out16 = torch.full((T, H, d), 5.0, dtype=torch.float16, device=DEV)
    out32 = torch.full((T, H, d), 5.0, dtype=torch.float32, device=DEV)
    tt = torch.from_numpy(table).to(DEV)
    K.tq_dequant_paged(packed, norms, tpi, tc, bits, out16, block_table=tt)
    K.tq_dequant_paged(packed, norms, tpi, tc, bits, out32, block_table=tt)  # CUDA-core kernel
    torch.cuda.synchronize()
    g16, g32 = out16.float().cpu().numpy(), out32.cpu().numpy()
    for b in (3, 7):
        assert not g16[16 * b:16 * b + 16].any() and not g32[16 * b:16 * b + 16].any()
    ops.assert_close_fp(g16, g32, rel=3e-4, label="tensor-core vs CUDA-core dequant", dtype="f16")


# ── batched append / gather by slot map ──

@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("bits,d", [(4, 128), (3, 128), (2, 128), (4, 64)])
def test_slot_map_append_equals_per_sequence_appends(dt, bits, d):
    """Decode-style batch: 300 sequences each append one token at their own position (own block
    table) — one slot-mapped launch equals 300 per-sequence block-table launches byte for byte;
    slot -1 is skipped and counted; the slot-mapped gather returns the same values."""
    H, nseq, nblk_per = 8, 300, 4
    rng = np.random.default_rng(bits + d)
    pos = rng.integers(0, nblk_per * 16, nseq)
    tables_ = rng.permutation(nseq * nblk_per).astype(np.int32).reshape(nseq, nblk_per)
    slots = (tables_[np.arange(nseq), pos // 16].astype(np.int64) * 16 + pos % 16)
    slots[[7, 150]] = -1
    x, raw = make_input(nseq, H, d, dt, seed=9)
    pi, c = tables(d, bits, 777)
    tpi, tc = torch.from_numpy(pi).to(DEV), torch.from_numpy(c).to(DEV)
    P = tq.TurboQuantConfig.packed_dim_per_head(d, bits)
    rows = nseq * nblk_per * 16
    pk1 = torch.full((rows, H * P), 0x3C, dtype=torch.uint8, device=DEV)
    nr1 = torch.full((rows, H), 0x1234, dtype=torch.int16, device=DEV)
    pk2, nr2 = pk1.clone(), nr1.clone()
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    xd = dev(x, dt)
    K.tq_compress_slots(xd, tpi, tc, bits, pk1, nr1, torch.from_numpy(slots).to(DEV), err=err)
    for sq in range(nseq):
        if slots[sq] < 0:
            continue
        K.tq_compress_paged(xd[sq:sq + 1], tpi, tc, bits, pk2, nr2,
                            block_table=torch.from_numpy(tables_[sq]).to(DEV), start_pos=int(pos[sq]))
    torch.cuda.synchronize()
    assert err.item() == 2 * H  # counted once per head vector
    assert torch.equal(pk1, pk2) and torch.equal(nr1, nr2)
    # against the exact statement, row by row
    pc, nc, _ = tq.compress_c(raw, KIND[dt], pi, c, bits)
    ok = slots >= 0
    assert np.array_equal(pk1.cpu().numpy()[slots[ok]], pc[ok])
    assert np.array_equal(nr1.cpu().numpy().view(np.uint16)[slots[ok]], nc[ok])
    # gather back
    out = torch.full((nseq, H, d), 3.0, dtype=torch.float16, device=DEV)
    K.tq_dequant_slots(pk1, nr1, tpi, tc, bits, out, torch.from_numpy(slots).to(DEV))
    torch.cuda.synchronize()
    got = out.float().cpu().numpy()
    assert not got[~ok].any()
    ref = tq.decompress_c(pc[ok], nc[ok], pi, c, bits, H, d).reshape(-1, H, d)
    ops.assert_close_fp(got[ok], ref, rel=3e-4, label="slot-mapped dequant", dtype="f16")
