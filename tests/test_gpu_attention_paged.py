"""Paged attention over the FP16/BF16 KV cache (fb_launch_attention_paged, launch_paged_attention)
and the paged append (fb_launch_kv_append_paged), against the float64 statement of the reference
kernel (``oracle.ops.attention_paged``, ``attention_paged.cu:25-159``) and the reference kernel
itself (``oracle/_ref``).

Bar (north star, FP16/BF16 outputs): max-abs error within 2e-3 of the output's magnitude beyond
the output dtype's rounding, cosine >= 0.9999. The append is a byte copy: bit-exact.
"""

import ctypes as C
from pathlib import Path

import numpy as np
import pytest
import torch

from fracture_b200 import _lib
from fracture_b200 import kernels as K
from oracle import ops

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
D = 128
TDT = {"f16": torch.float16, "bf16": torch.bfloat16}
REF_SO = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libfracture_ref_kernels.so"


def build_cache(kv_lens, Hkv, dt, seed, appends=3):
    """Shared pools; sequence s owns ceil(kv_lens[s] / 16) shuffled blocks, written by
    fb_launch_kv_append_paged in `appends` uneven pieces."""
    rng = np.random.default_rng(seed)
    nblk = [(L + 15) // 16 for L in kv_lens]
    total = sum(nblk) + 2
    perm = rng.permutation(total).astype(np.int32)
    max_blocks = max(nblk + [1])
    tables = np.full((len(kv_lens), max_blocks), -1, np.int32)
    k = 0
    for s, n in enumerate(nblk):
        tables[s, :n] = perm[k:k + n]
        k += n
    rows = total * 16
    kp = torch.full((rows, Hkv, D), 9.0, dtype=TDT[dt], device=DEV)
    vp = torch.full((rows, Hkv, D), 9.0, dtype=TDT[dt], device=DEV)
    host_k = np.full((rows, Hkv, D), 9.0)
    host_v = np.full((rows, Hkv, D), 9.0)
    for s, L in enumerate(kv_lens):
        kx = ops.round_to(rng.standard_normal((L, Hkv, D)) * 1.5, dt)
        vx = ops.round_to(rng.standard_normal((L, Hkv, D)), dt)
        bt = torch.from_numpy(tables[s]).to(DEV)
        cuts = sorted(set([0, L] + list(rng.integers(0, L + 1, appends - 1)))) if L else [0, 0]
        for a, b in zip(cuts[:-1], cuts[1:]):
            if b > a:
                K.kv_append_paged(torch.from_numpy(kx[a:b]).to(DEV).to(TDT[dt]),
                                  torch.from_numpy(vx[a:b]).to(DEV).to(TDT[dt]), kp, vp, bt, start_pos=a)
        pos = np.arange(L)
        sl = tables[s][pos // 16] * 16 + pos % 16
        host_k[sl], host_v[sl] = kx, vx
    torch.cuda.synchronize()
    return {"kp": kp, "vp": vp, "hk": host_k, "hv": host_v, "tables": tables, "Hkv": Hkv, "dt": dt}


def make_q(S, Tq, Hq, dt, seed):
    x = ops.round_to(np.random.default_rng(seed).standard_normal((S, Tq, Hq, D)), dt)
    return x, torch.from_numpy(x).to(DEV).to(TDT[dt])


def run_ours(c, q, kv_lens, starts):
    out = torch.full(q.shape, 7.0, dtype=q.dtype, device=DEV)
    K.attention_paged(q, c["kp"], c["vp"], torch.from_numpy(c["tables"]).to(DEV),
                      torch.tensor(kv_lens, dtype=torch.int32, device=DEV),
                      torch.tensor(starts, dtype=torch.int32, device=DEV), out)
    torch.cuda.synchronize()
    return out


def test_append_places_rows_through_the_block_table():
    c = build_cache([45, 300], 8, "f16", seed=1, appends=4)
    assert np.array_equal(c["kp"].float().cpu().numpy(), c["hk"])
    assert np.array_equal(c["vp"].float().cpu().numpy(), c["hv"])


def test_append_skips_missing_blocks_and_counts_them():
    Hkv = 2
    kp = torch.zeros((32, Hkv, D), dtype=torch.float16, device=DEV)
    vp = torch.zeros_like(kp)
    table = torch.tensor([1, -1], dtype=torch.int32, device=DEV)
    x = torch.ones((20, Hkv, D), dtype=torch.float16, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    K.kv_append_paged(x, x, kp, vp, table, start_pos=0, err=err)
    torch.cuda.synchronize()
    assert err.item() == 4  # tokens 16..19: no block
    assert kp[16:32].eq(1).all() and not kp[:16].any()


@pytest.mark.parametrize("G,dt", [(4, "f16"), (1, "f16"), (2, "bf16"), (8, "bf16")])
def test_decode_matches_statement(G, dt):
    Hkv = 2
    kv_lens = [1, 257, 900]
    c = build_cache(kv_lens, Hkv, dt, seed=G)
    qh, q = make_q(3, 1, G * Hkv, dt, seed=10 + G)
    starts = [L - 1 for L in kv_lens]
    got = run_ours(c, q, kv_lens, starts).float().cpu().numpy()
    for s, L in enumerate(kv_lens):
        ref = ops.attention_paged(qh[s], c["hk"], c["hv"], c["tables"][s], L, starts[s])
        ops.assert_close_fp(got[s], ref, rel=2e-3, min_cos=0.9999, label=f"seq {s}", dtype=dt)


def test_prefill_chunk_causal_and_missing_block():
    kv_lens, Tq, Hkv, G = [33, 700], 6, 2, 4
    c = build_cache(kv_lens, Hkv, "f16", seed=5)
    c["tables"][1, 4] = -1
    qh, q = make_q(2, Tq, G * Hkv, "f16", seed=6)
    starts = [L - Tq for L in kv_lens]
    got = run_ours(c, q, kv_lens, starts).float().cpu().numpy()
    for s, L in enumerate(kv_lens):
        ref = ops.attention_paged(qh[s], c["hk"], c["hv"], c["tables"][s], L, starts[s])
        ops.assert_close_fp(got[s], ref, rel=2e-3, min_cos=0.9999, label=f"seq {s}", dtype="f16")


def _reference_abi(lib, c, q, kv_len, start):
    Tq, Hq, _ = q.shape
    Hkv = c["Hkv"]
    nblocks = int(c["tables"].max()) + 1
    stride = 16 * Hkv * D * 2
    kptr = torch.tensor([c["kp"].data_ptr() + b * stride for b in range(nblocks)], dtype=torch.int64, device=DEV)
    vptr = torch.tensor([c["vp"].data_ptr() + b * stride for b in range(nblocks)], dtype=torch.int64, device=DEV)
    nb = (kv_len + 15) // 16
    bt = torch.from_numpy(np.ascontiguousarray(c["tables"][0][:nb])).to(DEV)
    out = torch.full((Tq, Hq, D), 7.0, dtype=torch.float16, device=DEV)
    rc = lib.launch_paged_attention(out.data_ptr(), q.data_ptr(), bt.data_ptr(), kptr.data_ptr(), vptr.data_ptr(), Tq,
                                    Hq, Hkv, D, kv_len, start, nb, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0
    return out


def test_reference_abi_equals_batched_entry():
    kv_len, Tq, Hkv, G = 600, 3, 2, 4
    c = build_cache([kv_len], Hkv, "f16", seed=7)
    qh, q = make_q(1, Tq, G * Hkv, "f16", seed=8)
    ours = run_ours(c, q, [kv_len], [kv_len - Tq])
    abi = _reference_abi(_lib.load(), c, q[0], kv_len, kv_len - Tq)
    assert torch.equal(abi, ours[0])


def test_reference_kernel_meets_the_bar_against_the_statement():
    """The reference's own kernel (oracle/_ref, fast-math) on the same cache and queries."""
    if not REF_SO.exists():
        pytest.skip("oracle/_ref not built (make -C oracle ref needs the reference sources)")
    ref = C.CDLL(str(REF_SO))
    ref.launch_paged_attention.argtypes = [C.c_void_p] * 5 + [C.c_int] * 7 + [C.c_void_p]
    ref.launch_paged_attention.restype = C.c_int
    kv_len, Tq, Hkv, G = 400, 2, 2, 4
    c = build_cache([kv_len], Hkv, "f16", seed=9)
    qh, q = make_q(1, Tq, G * Hkv, "f16", seed=10)
    got = _reference_abi(ref, c, q[0], kv_len, kv_len - Tq).float().cpu().numpy()
    ops.assert_close_fp(got, ops.attention_paged(qh[0], c["hk"], c["hv"], c["tables"][0], kv_len, kv_len - Tq),
                        rel=2e-3, min_cos=0.9999, label="reference kernel", dtype="f16")


def test_chunk_boundaries_and_more_items_than_ctas():
    """Contexts at and around the 512-position chunk edge and several chunks long, 40 prefill
    query tokens per sequence: more (chunk, KV head, token) items than the persistent grid has
    CTAs."""
    kv_lens, Tq, Hkv, G = [511, 512, 513, 1537], 40, 2, 4
    c = build_cache(kv_lens, Hkv, "bf16", seed=11)
    qh, q = make_q(len(kv_lens), Tq, G * Hkv, "bf16", seed=12)
    starts = [L - Tq for L in kv_lens]
    got = run_ours(c, q, kv_lens, starts).float().cpu().numpy()
    for s, L in enumerate(kv_lens):
        ref = ops.attention_paged(qh[s], c["hk"], c["hv"], c["tables"][s], L, starts[s])
        ops.assert_close_fp(got[s], ref, rel=2e-3, min_cos=0.9999, label=f"seq {s} (kv {L})", dtype="bf16")


def _rounds(max_kv_len, hkv, rows, sms):
    """Rounds of four 16-position tiles per warp and work item that the tensor-core attention
    kernels pick for a call (tc_chunks): 4, halved while the call's items would fill less than
    three quarters of a wave of two CTAs per SM."""
    positions = -(-max_kv_len // 256) * 256
    rnd = 4
    while rnd > 1 and -(-positions // (512 * rnd)) * hkv * rows * 4 < 6 * sms:
        rnd //= 2
    return rnd


def _queries_for_rounds(target, kv_lens, hkv):
    """A query count per sequence for which this GPU's SM count makes the kernel take `target` rounds."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    for tq in range(1, min(kv_lens) + 1):
        if _rounds(max(kv_lens), hkv, len(kv_lens) * tq, sms) == target:
            return tq
    pytest.skip(f"no query count gives {target} rounds on {sms} SMs")


@pytest.mark.parametrize("rnd", [1, 2, 4])
def test_ragged_contexts_at_every_item_length(rnd):
    """Ragged contexts around tile and item edges (513, 1040, 1064, 2100 positions), with the query
    count per sequence chosen from this GPU's SM count so that the tensor-core kernel takes items
    of 1, 2 and 4 rounds (512, 1024 and 2048 positions): every item length ends in a partial item
    whose later rounds are empty for some warps."""
    kv_lens, Hkv, G = [513, 1040, 1064, 2100], 2, 4
    Tq = _queries_for_rounds(rnd, kv_lens, Hkv)
    c = build_cache(kv_lens, Hkv, "f16", seed=70 + rnd)
    qh, q = make_q(len(kv_lens), Tq, G * Hkv, "f16", seed=71 + rnd)
    starts = [L - Tq for L in kv_lens]
    got = run_ours(c, q, kv_lens, starts).float().cpu().numpy()
    for s, L in enumerate(kv_lens):
        ref = ops.attention_paged(qh[s], c["hk"], c["hv"], c["tables"][s], L, starts[s])
        ops.assert_close_fp(got[s], ref, rel=2e-3, min_cos=0.9999, label=f"rnd {rnd}, seq {s} (kv {L})", dtype="f16")

def test_unaligned_queries_take_the_cuda_core_kernel():
    """Queries that do not start on a 16-byte boundary go through the CUDA-core kernel (the
    tensor-core kernel reads them 16 bytes at a time); both meet the bar."""
    kv_lens, Hkv, G = [300, 700], 2, 4
    c = build_cache(kv_lens, Hkv, "f16", seed=13)
    qh, q = make_q(2, 1, G * Hkv, "f16", seed=14)
    buf = torch.empty(q.numel() + 1, dtype=q.dtype, device=DEV)
    q_odd = buf[1:].view(q.shape)
    q_odd.copy_(q)
    assert q_odd.data_ptr() % 16 != 0
    starts = [L - 1 for L in kv_lens]
    for qq in (q, q_odd):
        got = run_ours(c, qq, kv_lens, starts).float().cpu().numpy()
        for s, L in enumerate(kv_lens):
            ref = ops.attention_paged(qh[s], c["hk"], c["hv"], c["tables"][s], L, starts[s])
            ops.assert_close_fp(got[s], ref, rel=2e-3, min_cos=0.9999, label=f"seq {s}", dtype="f16")


def test_pool_ending_inside_a_block_leaves_the_missing_rows_out():
    """Pools cut 5 rows into the last block a sequence uses: positions whose pool row lies past
    the pool are left out (as a missing block's are), on the tensor-core and CUDA-core kernels."""
    kv_lens, Hkv, G = [200], 2, 4
    c = build_cache(kv_lens, Hkv, "f16", seed=15)
    table = c["tables"][0]
    last = int(table.max())
    cut = last * 16 + 11  # rows last*16 + 11 .. last*16 + 15 are outside the pool
    qh, q = make_q(1, 1, G * Hkv, "f16", seed=16)
    pos = np.arange(kv_lens[0])
    rows = table[pos // 16] * 16 + pos % 16
    keep = rows < cut
    assert 0 < (~keep).sum() < len(pos)
    # expected: plain attention over the kept positions
    k, v = c["hk"][rows][keep], c["hv"][rows][keep]
    exp = np.zeros((1, G * Hkv, D))
    for h in range(G * Hkv):
        sc = k[:, h // G] @ qh[0, 0, h] / np.sqrt(D)
        p = np.exp(sc - sc.max())
        exp[0, h] = (p / p.sum()) @ v[:, h // G]
    for qq in (q, torch.empty(q.numel() + 1, dtype=q.dtype, device=DEV)[1:].view(q.shape).copy_(q)):
        out = torch.full(qq.shape, 7.0, dtype=qq.dtype, device=DEV)
        K.attention_paged(qq, c["kp"][:cut], c["vp"][:cut], torch.from_numpy(c["tables"]).to(DEV),
                          torch.tensor(kv_lens, dtype=torch.int32, device=DEV),
                          torch.tensor([kv_lens[0] - 1], dtype=torch.int32, device=DEV), out)
        torch.cuda.synchronize()
        ops.assert_close_fp(out[0].float().cpu().numpy(), exp, rel=2e-3, min_cos=0.9999, label="cut pool",
                            dtype="f16")
