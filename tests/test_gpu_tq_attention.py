"""TurboQuant paged attention against the float64 statement of the reference kernel
(``oracle.turboquant.attention_paged_tq``, ``attention_paged_tq.cu:56-259``) and against the
reference kernel itself (``oracle/_ref``), on caches written by this library's compress.

Bar (north star, FP16/BF16 outputs): max-abs error within 2e-3 of the output's magnitude
beyond the output dtype's rounding, cosine >= 0.9999. Both entry points run the same float32
kernels, so they agree bit for bit with each other.
"""

import ctypes as C
from pathlib import Path

import numpy as np
import pytest
import torch

from fracture_b200 import _lib
from fracture_b200 import kernels as K
from oracle import ops, turboquant as tq

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
D = 128
TDT = {"f16": torch.float16, "bf16": torch.bfloat16}
REF_SO = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libfracture_ref_kernels.so"


def build_cache(kv_lens, Hkv, kb, vb, seed):
    """Pools shared by the sequences; sequence s owns ceil(kv_lens[s] / 16) shuffled blocks,
    filled by fb_launch_tq_compress_paged with random keys and values."""
    rng = np.random.default_rng(seed)
    nblk = [(L + 15) // 16 for L in kv_lens]
    total = sum(nblk) + 3
    perm = rng.permutation(total).astype(np.int32)
    max_blocks = max(nblk + [1])
    tables = np.full((len(kv_lens), max_blocks), -1, np.int32)
    k = 0
    for s, n in enumerate(nblk):
        tables[s, :n] = perm[k:k + n]
        k += n
    rows = total * 16
    Pk, Pv = D * kb // 8, D * vb // 8
    c = {"kp": torch.zeros((rows, Hkv * Pk), dtype=torch.uint8, device=DEV),
         "vp": torch.zeros((rows, Hkv * Pv), dtype=torch.uint8, device=DEV),
         "kn": torch.zeros((rows, Hkv), dtype=torch.float16, device=DEV),
         "vn": torch.zeros((rows, Hkv), dtype=torch.float16, device=DEV)}
    pik, piv = K.tq_rotation_matrix(D, seed), K.tq_rotation_matrix(D, seed + 500)
    ck, cv = K.tq_codebook(D, kb)[0], K.tq_codebook(D, vb)[0]
    dev = {n: torch.from_numpy(np.ascontiguousarray(x)).to(DEV) for n, x in
           (("pik", pik), ("piv", piv), ("ck", ck), ("cv", cv))}
    for s, L in enumerate(kv_lens):
        if L == 0:
            continue
        kx = torch.from_numpy((rng.standard_normal((L, Hkv, D)) * 1.5).astype(np.float32)).to(DEV).half()
        vx = torch.from_numpy(rng.standard_normal((L, Hkv, D)).astype(np.float32)).to(DEV).half()
        bt = torch.from_numpy(tables[s]).to(DEV)
        K.tq_compress_paged(kx, dev["pik"], dev["ck"], kb, c["kp"], c["kn"], block_table=bt)
        K.tq_compress_paged(vx, dev["piv"], dev["cv"], vb, c["vp"], c["vn"], block_table=bt)
    torch.cuda.synchronize()
    c.update(dev)
    c.update({"tables": tables, "pik_h": pik, "piv_h": piv, "ck_h": ck, "cv_h": cv, "kb": kb, "vb": vb,
              "Hkv": Hkv})
    return c


def statement(c, q, s, kv_len, start):
    """The oracle for sequence s (q: [Tq, Hq, D] values)."""
    return tq.attention_paged_tq(q, c["kp"].cpu().numpy(), c["kn"].float().cpu().numpy(), c["vp"].cpu().numpy(),
                                 c["vn"].float().cpu().numpy(), c["tables"][s], kv_len, start, c["pik_h"],
                                 c["piv_h"], c["ck_h"], c["cv_h"], c["kb"], c["vb"], c["Hkv"])


def run_ours(c, q, kv_lens, starts, dt):
    S, Tq, Hq, _ = q.shape
    out = torch.full(q.shape, 7.0, dtype=TDT[dt], device=DEV)
    K.tq_attention_paged(q, c["kp"], c["kn"], c["vp"], c["vn"], torch.from_numpy(c["tables"]).to(DEV),
                         torch.tensor(kv_lens, dtype=torch.int32, device=DEV),
                         torch.tensor(starts, dtype=torch.int32, device=DEV), c["pik"], c["piv"], c["ck"], c["cv"],
                         c["kb"], c["vb"], out)
    torch.cuda.synchronize()
    return out


def make_q(S, Tq, Hq, dt, seed):
    x = np.random.default_rng(seed).standard_normal((S, Tq, Hq, D)).astype(np.float32)
    x = ops.round_to(x, dt)
    return x, torch.from_numpy(x).to(DEV).to(TDT[dt])


@pytest.mark.parametrize("G,kb,vb,dt", [(4, 4, 2, "f16"), (1, 4, 4, "f16"), (2, 3, 3, "bf16"), (8, 8, 8, "f16"),
                                        (4, 2, 4, "bf16"), (8, 4, 2, "bf16"), (2, 2, 2, "f16"), (4, 3, 2, "f16")])
def test_decode_matches_statement(G, kb, vb, dt):
    """One query token per sequence at the end of its context (decode), contexts of 1 to 777
    positions (one to four 256-position chunks of the CUDA-core kernel, one or two 512-position
    chunks of the tensor-core kernel, which takes short items for small batches), GQA groups of
    1 to 8."""
    Hkv = 2
    kv_lens = [1, 300, 777]
    c = build_cache(kv_lens, Hkv, kb, vb, seed=10 * G + kb)
    qh, q = make_q(len(kv_lens), 1, G * Hkv, dt, seed=G + vb)
    starts = [L - 1 for L in kv_lens]
    got = run_ours(c, q, kv_lens, starts, dt).float().cpu().numpy()
    for s, L in enumerate(kv_lens):
        ref = statement(c, qh[s], s, L, starts[s])
        ops.assert_close_fp(got[s], ref, rel=2e-3, min_cos=0.9999, label=f"seq {s} (kv {L})", dtype=dt)


def test_prefill_chunk_causal():
    """Seven query tokens per sequence appended at the end: token t sees start + t + 1 positions."""
    kv_lens, Tq, Hkv, G = [40, 600], 7, 2, 4
    c = build_cache(kv_lens, Hkv, 4, 2, seed=3)
    qh, q = make_q(2, Tq, G * Hkv, "f16", seed=4)
    starts = [L - Tq for L in kv_lens]
    got = run_ours(c, q, kv_lens, starts, "f16").float().cpu().numpy()
    for s, L in enumerate(kv_lens):
        ops.assert_close_fp(got[s], statement(c, qh[s], s, L, starts[s]), rel=2e-3, min_cos=0.9999,
                            label=f"seq {s}", dtype="f16")


def test_missing_block_and_empty_sequence():
    """A negative block-table entry leaves its 16 positions out; a sequence with no positions
    gives zeros."""
    kv_lens, Hkv, G = [0, 90, 513], 2, 4
    c = build_cache(kv_lens, Hkv, 4, 2, seed=8)
    c["tables"][2, 3] = -1
    c["tables"][1, 0] = -1
    qh, q = make_q(3, 1, G * Hkv, "f16", seed=9)
    starts = [max(L - 1, 0) for L in kv_lens]
    got = run_ours(c, q, kv_lens, starts, "f16").float().cpu().numpy()
    assert not np.any(got[0])
    for s in (1, 2):
        ops.assert_close_fp(got[s], statement(c, qh[s], s, kv_lens[s], starts[s]), rel=2e-3, min_cos=0.9999,
                            label=f"seq {s}", dtype="f16")


def _block_pointer_arrays(c, nblocks):
    Hkv = c["Hkv"]
    Pk, Pv = D * c["kb"] // 8, D * c["vb"] // 8
    arr = lambda base, stride: torch.tensor([base + b * 16 * stride for b in range(nblocks)], dtype=torch.int64,
                                            device=DEV)
    return (arr(c["kp"].data_ptr(), Hkv * Pk), arr(c["kn"].data_ptr(), Hkv * 2), arr(c["vp"].data_ptr(), Hkv * Pv),
            arr(c["vn"].data_ptr(), Hkv * 2))


def _reference_abi_call(lib, c, q, kv_len, start):
    Tq, Hq, _ = q.shape
    nblocks = int(c["tables"].max()) + 1
    kp, kn, vp, vn = _block_pointer_arrays(c, nblocks)
    bt = torch.from_numpy(np.ascontiguousarray(c["tables"][0])).to(DEV)
    out = torch.full((Tq, Hq, D), 7.0, dtype=torch.float16, device=DEV)
    Pk, Pv = D * c["kb"] // 8, D * c["vb"] // 8
    rc = lib.launch_attention_paged_tq(out.data_ptr(), q.data_ptr(), bt.data_ptr(), kp.data_ptr(), kn.data_ptr(),
                                       vp.data_ptr(), vn.data_ptr(), c["pik"].data_ptr(), c["piv"].data_ptr(),
                                       c["ck"].data_ptr(), c["cv"].data_ptr(), Tq, Hq, c["Hkv"], D, kv_len, start,
                                       c["kb"], c["vb"], Pk, Pv, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0
    return out


@pytest.mark.parametrize("kb,vb", [(4, 2), (8, 8), (2, 4)])
def test_reference_abi_equals_batched_entry(kb, vb):
    """launch_attention_paged_tq (per-block pointer arrays, ffi.rs:251-274) gives the batched entry
    point's result bit for bit, and both meet the bar against the statement."""
    kv_len, Tq, Hkv, G = 700, 3, 2, 4
    c = build_cache([kv_len], Hkv, kb, vb, seed=20 + kb)
    qh, q = make_q(1, Tq, G * Hkv, "f16", seed=21)
    ours = run_ours(c, q, [kv_len], [kv_len - Tq], "f16")
    abi = _reference_abi_call(_lib.load(), c, q[0], kv_len, kv_len - Tq)
    assert torch.equal(abi, ours[0])
    ops.assert_close_fp(abi.float().cpu().numpy(), statement(c, qh[0], 0, kv_len, kv_len - Tq), rel=2e-3,
                        min_cos=0.9999, label="reference ABI", dtype="f16")


@pytest.mark.parametrize("kb,vb", [(4, 2), (4, 4), (2, 2), (8, 8)])
def test_reference_kernel_meets_the_bar_against_the_statement(kb, vb):
    """The reference's own kernel (oracle/_ref, fast-math) on the same cache and queries: within
    the bar of the float64 statement, which pins the oracle to the reference implementation."""
    if not REF_SO.exists():
        pytest.skip("oracle/_ref not built (make -C oracle ref needs the reference sources)")
    ref = C.CDLL(str(REF_SO))
    ref.launch_attention_paged_tq.argtypes = [C.c_void_p] * 11 + [C.c_int] * 10 + [C.c_void_p]
    ref.launch_attention_paged_tq.restype = C.c_int
    kv_len, Tq, Hkv, G = 400, 2, 2, 4
    c = build_cache([kv_len], Hkv, kb, vb, seed=40 + kb + vb)
    qh, q = make_q(1, Tq, G * Hkv, "f16", seed=41)
    got = _reference_abi_call(ref, c, q[0], kv_len, kv_len - Tq).float().cpu().numpy()
    ops.assert_close_fp(got, statement(c, qh[0], 0, kv_len, kv_len - Tq), rel=2e-3, min_cos=0.9999,
                        label="reference kernel", dtype="f16")


@pytest.mark.parametrize("kb,vb", [(4, 2), (2, 2)])
def test_chunk_boundaries_and_more_items_than_ctas(kb, vb):
    """Contexts crossing several chunk edges of the tensor-core kernel (512-position items at this
    batch size; the full-size tests cover the longer ones), with 40 prefill query tokens per
    sequence: more (chunk, KV head, token) items than the persistent grid has CTAs, so CTAs take
    several each."""
    kv_lens, Tq, Hkv, G = [513, 1040, 1064, 2100], 40, 2, 4
    c = build_cache(kv_lens, Hkv, kb, vb, seed=60 + kb + vb)
    qh, q = make_q(len(kv_lens), Tq, G * Hkv, "f16", seed=61)
    starts = [L - Tq for L in kv_lens]
    got = run_ours(c, q, kv_lens, starts, "f16").float().cpu().numpy()
    for s, L in enumerate(kv_lens):
        ops.assert_close_fp(got[s], statement(c, qh[s], s, L, starts[s]), rel=2e-3, min_cos=0.9999,
                            label=f"seq {s} (kv {L})", dtype="f16")


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
def test_per_head_kernel_ragged_contexts_at_every_item_length(rnd):
    """The per-head tensor-core kernel (2 KV heads, 4-bit keys, 2-bit values) on ragged contexts
    (513, 1040, 1064, 2100 positions), with the query count per sequence chosen from this GPU's SM
    count so that it takes items of 1, 2 and 4 rounds (512, 1024 and 2048 positions): every item
    length ends in a partial item."""
    kv_lens, Hkv, G, kb, vb = [513, 1040, 1064, 2100], 2, 4, 4, 2
    Tq = _queries_for_rounds(rnd, kv_lens, Hkv)
    c = build_cache(kv_lens, Hkv, kb, vb, seed=80 + rnd)
    qh, q = make_q(len(kv_lens), Tq, G * Hkv, "f16", seed=81 + rnd)
    starts = [L - Tq for L in kv_lens]
    before = K.tq_path_counts()["attention_per_head"]
    got = run_ours(c, q, kv_lens, starts, "f16").float().cpu().numpy()
    assert K.tq_path_counts()["attention_per_head"] == before + 1
    for s, L in enumerate(kv_lens):
        ops.assert_close_fp(got[s], statement(c, qh[s], s, L, starts[s]), rel=2e-3, min_cos=0.9999,
                            label=f"rnd {rnd}, seq {s} (kv {L})", dtype="f16")

@pytest.mark.parametrize("kb,vb", [(4, 2), (3, 3)])
def test_pool_ending_inside_a_block_leaves_the_missing_rows_out(kb, vb):
    """Pools cut 5 rows into the last block the sequence uses: positions whose pool row lies past
    the pool are left out (the tensor-core kernel for 4/2 bits, the CUDA-core one for 3/3)."""
    kv_len, Hkv, G = 200, 2, 4
    c = build_cache([kv_len], Hkv, kb, vb, seed=70 + kb)
    table = c["tables"][0]
    last = int(table.max())
    cut = last * 16 + 11
    qh, q = make_q(1, 1, G * Hkv, "f16", seed=71)
    # expected: the statement over a cache whose cut rows hold no block (their block entry
    # stays, but the statement sees the kept positions only through a per-position table)
    pos = np.arange(kv_len)
    rows = table[pos // 16] * 16 + pos % 16
    keep = rows < cut
    assert 0 < (~keep).sum() < kv_len
    d = D
    Pk, Pv = d * kb // 8, d * vb // 8
    kp = c["kp"].cpu().numpy().reshape(-1, Hkv, Pk)[rows[keep]]
    vp = c["vp"].cpu().numpy().reshape(-1, Hkv, Pv)[rows[keep]]
    kn = c["kn"].float().cpu().numpy()[rows[keep]]
    vn = c["vn"].float().cpu().numpy()[rows[keep]]
    n = int(keep.sum())
    nb = (n + 15) // 16
    pad = nb * 16 - n
    kp = np.concatenate([kp, np.zeros((pad, Hkv, Pk), np.uint8)]).reshape(nb * 16, Hkv * Pk)
    vp = np.concatenate([vp, np.zeros((pad, Hkv, Pv), np.uint8)]).reshape(nb * 16, Hkv * Pv)
    kn = np.concatenate([kn, np.zeros((pad, Hkv))])
    vn = np.concatenate([vn, np.zeros((pad, Hkv))])
    exp = tq.attention_paged_tq(qh[0], kp, kn, vp, vn, np.arange(nb), n, n - 1, c["pik_h"], c["piv_h"], c["ck_h"],
                                c["cv_h"], kb, vb, Hkv)
    out = torch.full(q.shape, 7.0, dtype=torch.float16, device=DEV)
    K.tq_attention_paged(q, c["kp"][:cut], c["kn"][:cut], c["vp"][:cut], c["vn"][:cut],
                         torch.from_numpy(c["tables"]).to(DEV), torch.tensor([kv_len], dtype=torch.int32, device=DEV),
                         torch.tensor([kv_len - 1], dtype=torch.int32, device=DEV), c["pik"], c["piv"], c["ck"],
                         c["cv"], kb, vb, out)
    torch.cuda.synchronize()
    ops.assert_close_fp(out[0].float().cpu().numpy(), exp, rel=2e-3, min_cos=0.9999, label="cut pool", dtype="f16")


def test_reference_abi_calls_on_two_streams_at_once():
    """launch_attention_paged_tq keeps one library workspace per device and stream: calls queued
    alternately on two streams (free to overlap on the GPU) give the same bytes as calls made
    one after the other."""
    kv_len, Tq, Hkv, G = 3000, 4, 2, 4
    c = build_cache([kv_len], Hkv, 4, 2, seed=80)
    lib = _lib.load()
    qs = [make_q(1, Tq, G * Hkv, "f16", seed=81 + i)[1][0] for i in range(4)]
    ref = [_reference_abi_call(lib, c, qq, kv_len, kv_len - Tq) for qq in qs]
    nblocks = int(c["tables"].max()) + 1
    kp, kn, vp, vn = _block_pointer_arrays(c, nblocks)
    bt = torch.from_numpy(np.ascontiguousarray(c["tables"][0])).to(DEV)
    outs = [torch.full_like(r, 7.0) for r in ref]
    torch.cuda.synchronize()  # everything above is ready before the streams start
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    Hq = G * Hkv
    for _ in range(3):
        for i, qq in enumerate(qs):
            rc = lib.launch_attention_paged_tq(outs[i].data_ptr(), qq.data_ptr(), bt.data_ptr(), kp.data_ptr(),
                                               kn.data_ptr(), vp.data_ptr(), vn.data_ptr(), c["pik"].data_ptr(),
                                               c["piv"].data_ptr(), c["ck"].data_ptr(), c["cv"].data_ptr(), Tq, Hq,
                                               Hkv, D, kv_len, kv_len - Tq, 4, 2, D // 2, D // 4,
                                               streams[i % 2].cuda_stream)
            assert rc == 0
    torch.cuda.synchronize()
    for o, r in zip(outs, ref):
        assert torch.equal(o, r)


# ── the streamed tensor-core kernel (pool-backed caches, KV heads a multiple of 8) ──

def _run_counted(path, fn):
    """fn() and whether exactly one call of it was served by the named attention path."""
    before = K.tq_path_counts()[path]
    out = fn()
    return out, K.tq_path_counts()[path] - before


@pytest.mark.parametrize("G,kb,vb,dt", [(4, 4, 2, "f16"), (1, 4, 4, "f16"), (2, 2, 2, "bf16"), (8, 2, 4, "f16"),
                                        (4, 4, 4, "bf16"), (4, 8, 8, "f16"), (2, 8, 4, "bf16"), (4, 2, 8, "f16"),
                                        (8, 8, 2, "f16")])
def test_streamed_kernel_decode_matches_statement(G, kb, vb, dt):
    """Eight KV heads (one head group): decode at contexts that end inside a stage, cross chunk
    edges and take an item to its last stage, for each bit-width pair (8-bit codes included: the
    reference's protected layers), group size and query dtype."""
    kv_lens, Hkv = [300, 777, 1500, 2049], 8
    c = build_cache(kv_lens, Hkv, kb, vb, seed=100 + 10 * G + kb + vb)
    qh, q = make_q(len(kv_lens), 1, G * Hkv, dt, seed=101 + G)
    starts = [L - 1 for L in kv_lens]
    got, served = _run_counted("attention_streamed", lambda: run_ours(c, q, kv_lens, starts, dt))
    assert served == 1
    got = got.float().cpu().numpy()
    for s, L in enumerate(kv_lens):
        ops.assert_close_fp(got[s], statement(c, qh[s], s, L, starts[s]), rel=2e-3, min_cos=0.9999,
                            label=f"seq {s} (kv {L})", dtype=dt)


@pytest.mark.parametrize("kb,vb", [(4, 2), (8, 8)])
def test_streamed_kernel_prefill_chunk_causal_and_many_items(kb, vb):
    """40 query tokens per sequence with their own causal ranges (the tokens of a sequence share
    a chunk's codes), more items than the persistent grid has CTAs."""
    kv_lens, Tq, Hkv, G = [60, 600, 1100, 2100], 40, 8, 4
    c = build_cache(kv_lens, Hkv, kb, vb, seed=110 + kb)
    qh, q = make_q(len(kv_lens), Tq, G * Hkv, "f16", seed=111)
    starts = [L - Tq for L in kv_lens]
    got, served = _run_counted("attention_streamed", lambda: run_ours(c, q, kv_lens, starts, "f16"))
    assert served == 1
    got = got.float().cpu().numpy()
    for s, L in enumerate(kv_lens):
        ops.assert_close_fp(got[s], statement(c, qh[s], s, L, starts[s]), rel=2e-3, min_cos=0.9999,
                            label=f"seq {s} (kv {L})", dtype="f16")


def test_streamed_kernel_missing_blocks_and_empty_sequence():
    """Negative block-table entries (one in each block slot of a stage, and a first block) leave
    their positions out; an empty sequence gives zeros."""
    kv_lens, Hkv, G = [0, 90, 513, 1029], 8, 4
    c = build_cache(kv_lens, Hkv, 2, 2, seed=120)
    c["tables"][1, 0] = -1
    c["tables"][2, 3] = -1
    c["tables"][3, 10] = -1
    c["tables"][3, 11] = -1
    c["tables"][3, 40] = -1
    qh, q = make_q(len(kv_lens), 1, G * Hkv, "f16", seed=121)
    starts = [max(L - 1, 0) for L in kv_lens]
    got, served = _run_counted("attention_streamed", lambda: run_ours(c, q, kv_lens, starts, "f16"))
    assert served == 1
    got = got.float().cpu().numpy()
    assert not np.any(got[0])
    for s in (1, 2, 3):
        ops.assert_close_fp(got[s], statement(c, qh[s], s, kv_lens[s], starts[s]), rel=2e-3, min_cos=0.9999,
                            label=f"seq {s}", dtype="f16")


@pytest.mark.parametrize("kb,vb", [(4, 2), (8, 8)])
def test_streamed_kernel_pool_ending_inside_a_block(kb, vb):
    """A pool cut 5 rows into the last block the sequence uses: the kernel's copies read zeros
    past the pool's end, and the positions there are left out."""
    kv_len, Hkv, G = 700, 8, 4
    c = build_cache([kv_len], Hkv, kb, vb, seed=130 + kb)
    table = c["tables"][0]
    cut = int(table.max()) * 16 + 11
    qh, q = make_q(1, 1, G * Hkv, "f16", seed=131)
    pos = np.arange(kv_len)
    rows = table[pos // 16] * 16 + pos % 16
    keep = rows < cut
    assert 0 < (~keep).sum() < kv_len
    Pk, Pv = D * kb // 8, D * vb // 8
    n = int(keep.sum())
    nb = (n + 15) // 16
    pad = nb * 16 - n
    kp = np.concatenate([c["kp"].cpu().numpy().reshape(-1, Hkv, Pk)[rows[keep]],
                         np.zeros((pad, Hkv, Pk), np.uint8)]).reshape(nb * 16, Hkv * Pk)
    vp = np.concatenate([c["vp"].cpu().numpy().reshape(-1, Hkv, Pv)[rows[keep]],
                         np.zeros((pad, Hkv, Pv), np.uint8)]).reshape(nb * 16, Hkv * Pv)
    kn = np.concatenate([c["kn"].float().cpu().numpy()[rows[keep]], np.zeros((pad, Hkv))])
    vn = np.concatenate([c["vn"].float().cpu().numpy()[rows[keep]], np.zeros((pad, Hkv))])
    exp = tq.attention_paged_tq(qh[0], kp, kn, vp, vn, np.arange(nb), n, n - 1, c["pik_h"], c["piv_h"], c["ck_h"],
                                c["cv_h"], kb, vb, Hkv)
    out = torch.full(q.shape, 7.0, dtype=torch.float16, device=DEV)

    def call():
        K.tq_attention_paged(q, c["kp"][:cut], c["kn"][:cut], c["vp"][:cut], c["vn"][:cut],
                             torch.from_numpy(c["tables"]).to(DEV),
                             torch.tensor([kv_len], dtype=torch.int32, device=DEV),
                             torch.tensor([kv_len - 1], dtype=torch.int32, device=DEV), c["pik"], c["piv"], c["ck"],
                             c["cv"], kb, vb, out)
        torch.cuda.synchronize()

    _, served = _run_counted("attention_streamed", call)
    assert served == 1
    ops.assert_close_fp(out[0].float().cpu().numpy(), exp, rel=2e-3, min_cos=0.9999, label="cut pool", dtype="f16")


def test_streamed_kernel_two_head_groups():
    """Sixteen KV heads: two items per (chunk, token), one per group of eight, each reading its
    half of every pool row."""
    kv_lens, Tq, Hkv, G = [700, 1300], 3, 16, 2
    c = build_cache(kv_lens, Hkv, 4, 4, seed=140)
    qh, q = make_q(len(kv_lens), Tq, G * Hkv, "f16", seed=141)
    starts = [L - Tq for L in kv_lens]
    got, served = _run_counted("attention_streamed", lambda: run_ours(c, q, kv_lens, starts, "f16"))
    assert served == 1
    got = got.float().cpu().numpy()
    for s, L in enumerate(kv_lens):
        ops.assert_close_fp(got[s], statement(c, qh[s], s, L, starts[s]), rel=2e-3, min_cos=0.9999,
                            label=f"seq {s} (kv {L})", dtype="f16")


def test_short_contexts_stream_and_few_kv_heads_keep_the_per_head_kernel():
    """Contexts of at most 256 positions (one chunk) take the streamed kernel with 8 KV heads;
    KV-head counts that are not a multiple of 8 take the per-head tensor-core kernel."""
    for kv_lens, Hkv, path in (([200, 256, 17], 8, "attention_streamed"), ([900], 2, "attention_per_head")):
        c = build_cache(kv_lens, Hkv, 4, 2, seed=150 + Hkv)
        qh, q = make_q(len(kv_lens), 1, 4 * Hkv, "f16", seed=151)
        starts = [L - 1 for L in kv_lens]
        got, served = _run_counted(path, lambda: run_ours(c, q, kv_lens, starts, "f16"))
        assert served == 1
        got = got.float().cpu().numpy()
        for s, L in enumerate(kv_lens):
            ops.assert_close_fp(got[s], statement(c, qh[s], s, L, starts[s]), rel=2e-3, min_cos=0.9999,
                                label=f"Hkv {Hkv} seq {s}", dtype="f16")


def test_streamed_kernel_many_items_per_cta_and_ragged_lengths():
    """Forty sequences of 1000-3000 positions: several hundred items of different lengths, so
    every persistent CTA takes several (its stage ring and query prefetch run across them)."""
    rng = np.random.default_rng(160)
    kv_lens = [int(x) for x in rng.integers(1000, 3001, size=40)]
    Hkv, G = 8, 4
    c = build_cache(kv_lens, Hkv, 4, 2, seed=161)
    qh, q = make_q(len(kv_lens), 1, G * Hkv, "f16", seed=162)
    starts = [L - 1 for L in kv_lens]
    got, served = _run_counted("attention_streamed", lambda: run_ours(c, q, kv_lens, starts, "f16"))
    assert served == 1
    got = got.float().cpu().numpy()
    for s, L in enumerate(kv_lens):
        ops.assert_close_fp(got[s], statement(c, qh[s], s, L, starts[s]), rel=2e-3, min_cos=0.9999,
                            label=f"seq {s} (kv {L})", dtype="f16")


@pytest.mark.parametrize("kv_len,kb,vb", [(12000, 4, 2), (20000, 4, 2), (33000, 4, 2), (33000, 8, 8)])
def test_streamed_kernel_every_chunk_length(kv_len, kb, vb):
    """One long sequence: a row may have at most 32 partials, so these contexts take 512-, 1024-
    and 2048-position chunks (the last with 8-bit codes: 128 one-block stages per item), each
    ending inside a chunk and inside a stage."""
    Hkv, G = 8, 4
    c = build_cache([kv_len], Hkv, kb, vb, seed=170 + kv_len % 97 + kb)
    qh, q = make_q(1, 1, G * Hkv, "f16", seed=171)
    got, served = _run_counted("attention_streamed", lambda: run_ours(c, q, [kv_len], [kv_len - 1], "f16"))
    assert served == 1
    ops.assert_close_fp(got.float().cpu().numpy()[0], statement(c, qh[0], 0, kv_len, kv_len - 1), rel=2e-3,
                        min_cos=0.9999, label=f"kv {kv_len}", dtype="f16")


# ── the streamed kernel through the reference ABI (per-block buffers, ffi.rs:251-274) ──

def _scattered_block_buffers(c, nblocks, misalign):
    """Each block's code and norm rows copied to its own place in one buffer per tensor, as a
    cache of separate per-block allocations would hold them; with `misalign`, the odd blocks'
    codes start 1 byte and their norms 2 bytes past a 16-byte boundary. Returns the buffers
    (kept alive by the caller) and the four pointer arrays."""
    keep, arrays = [], []
    for name, shift in (("kp", 1), ("kn", 2), ("vp", 1), ("vn", 2)):
        flat = c[name].view(torch.uint8).reshape(-1)
        blk = flat.numel() // (c[name].shape[0] // 16)
        stride = (blk + 31) // 32 * 32 + 32
        buf = torch.zeros(nblocks * stride + 64, dtype=torch.uint8, device=DEV)
        ptrs = []
        for b in range(nblocks):
            off = b * stride + (shift if misalign and b % 2 else 0)
            buf[off:off + blk] = flat[b * blk:(b + 1) * blk]
            ptrs.append(buf.data_ptr() + off)
        keep.append(buf)
        arrays.append(torch.tensor(ptrs, dtype=torch.int64, device=DEV))
    return keep, arrays


def _abi_call(c, q, kv_len, start, arrays, table):
    """launch_attention_paged_tq on the given pointer arrays and block table (one sequence)."""
    lib = _lib.load()
    Tq, Hq, _ = q.shape
    kp, kn, vp, vn = arrays
    bt = torch.from_numpy(np.ascontiguousarray(table)).to(DEV)
    out = torch.full((Tq, Hq, D), 7.0, dtype=torch.float16, device=DEV)
    Pk, Pv = D * c["kb"] // 8, D * c["vb"] // 8
    rc = lib.launch_attention_paged_tq(out.data_ptr(), q.data_ptr(), bt.data_ptr(), kp.data_ptr(), kn.data_ptr(),
                                       vp.data_ptr(), vn.data_ptr(), c["pik"].data_ptr(), c["piv"].data_ptr(),
                                       c["ck"].data_ptr(), c["cv"].data_ptr(), Tq, Hq, c["Hkv"], D, kv_len, start,
                                       c["kb"], c["vb"], Pk, Pv, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0
    return out


@pytest.mark.parametrize("kb,vb,Hkv,Tq", [(4, 2, 8, 1), (8, 8, 8, 3), (2, 4, 8, 1), (4, 8, 8, 2), (8, 2, 8, 1),
                                          (4, 4, 16, 2), (2, 2, 16, 1)])
def test_reference_abi_streams_per_block_buffers(kb, vb, Hkv, Tq):
    """With a multiple of 8 KV heads the reference ABI takes the streamed kernel, its blocks'
    rows brought in by bulk copies from the per-block buffers (one per buffer with 8 KV heads,
    one per row with 16): the batched pool entry's result bit for bit (the same chunks and
    arithmetic), within the bar of the statement, over a context that ends inside a block."""
    kv_len, G = 1500, 4
    c = build_cache([kv_len], Hkv, kb, vb, seed=200 + kb + 3 * vb + Hkv)
    qh, q = make_q(1, Tq, G * Hkv, "f16", seed=201)
    ours = run_ours(c, q, [kv_len], [kv_len - Tq], "f16")
    arrays = _block_pointer_arrays(c, int(c["tables"].max()) + 1)
    abi, served = _run_counted("attention_streamed", lambda: _abi_call(c, q[0], kv_len, kv_len - Tq, arrays,
                                                                         c["tables"][0]))
    assert served == 1
    assert torch.equal(abi, ours[0])
    ops.assert_close_fp(abi.float().cpu().numpy(), statement(c, qh[0], 0, kv_len, kv_len - Tq), rel=2e-3,
                        min_cos=0.9999, label="reference ABI, streamed", dtype="f16")


@pytest.mark.parametrize("kb,vb,Hkv", [(4, 2, 8), (8, 8, 8), (4, 4, 16)])
def test_reference_abi_streams_misaligned_block_buffers(kb, vb, Hkv):
    """Per-block buffers in separate places, every other one not 16-byte aligned (codes 1 byte,
    norms 2 bytes off): those blocks are copied by the producer lanes without bulk copies, the
    others by bulk copies, within one call; a missing block (-1) is left out. Equal bit for bit
    to the pool entry on the same cache and table."""
    kv_len, Tq, G = 1100, 2, 4
    c = build_cache([kv_len], Hkv, kb, vb, seed=210 + kb + vb + Hkv)
    c["tables"][0, 5] = -1
    qh, q = make_q(1, Tq, G * Hkv, "f16", seed=211)
    ours = run_ours(c, q, [kv_len], [kv_len - Tq], "f16")
    keep, arrays = _scattered_block_buffers(c, c["kp"].shape[0] // 16, misalign=True)
    abi, served = _run_counted("attention_streamed", lambda: _abi_call(c, q[0], kv_len, kv_len - Tq, arrays,
                                                                         c["tables"][0]))
    assert served == 1
    assert torch.equal(abi, ours[0])
    ops.assert_close_fp(abi.float().cpu().numpy(), statement(c, qh[0], 0, kv_len, kv_len - Tq), rel=2e-3,
                        min_cos=0.9999, label="misaligned per-block buffers", dtype="f16")
    del keep


def _least_workspace(S, Tq, Hq, max_kv_len):
    """The least workspace the batched entry accepts: rotated queries and one partial per
    256-position chunk (fb_tq_attention_workspace_bytes gives more to calls with few rows)."""
    return S * Tq * Hq * (D * 4 + (D + 2) * 4 * ((max_kv_len + 255) // 256))


def test_workspace_sizing_gives_few_rows_finer_chunks():
    """fb_tq_attention_workspace_bytes: the least size for many rows, and up to one partial per
    32 positions (at most 160 per head over the rows) for few."""
    Hq = 32
    assert K.tq_attention_workspace_bytes(64, 1, Hq, 8192) == _least_workspace(64, 1, Hq, 8192)
    assert K.tq_attention_workspace_bytes(1, 1, Hq, 8192) == Hq * (D * 4 + (D + 2) * 4 * 160)
    assert K.tq_attention_workspace_bytes(1, 1, Hq, 1000) == Hq * (D * 4 + (D + 2) * 4 * 32)
    assert K.tq_attention_workspace_bytes(2, 1, Hq, 100000) == _least_workspace(2, 1, Hq, 100000)


@pytest.mark.parametrize("kv_lens,Tq,kb,vb", [([8192], 1, 4, 2), ([1000], 1, 2, 4), ([3000, 77], 2, 8, 8),
                                               ([20000], 1, 4, 4)])
def test_streamed_kernel_few_rows_split_finer(kv_lens, Tq, kb, vb):
    """Few query rows: the streamed kernel cuts the context into chunks as short as 32 positions
    (one stage) so that every SM has an item, up to 160 partials per head; the same call with the
    least workspace keeps 256-position or longer chunks. Both meet the bar against the statement."""
    Hkv, G = 8, 4
    c = build_cache(kv_lens, Hkv, kb, vb, seed=220 + kb + vb + len(kv_lens))
    qh, q = make_q(len(kv_lens), Tq, G * Hkv, "f16", seed=221)
    starts = [L - Tq for L in kv_lens]
    S, Hq, L = len(kv_lens), G * Hkv, max(kv_lens)
    for ws_bytes in (K.tq_attention_workspace_bytes(S, Tq, Hq, L), _least_workspace(S, Tq, Hq, L)):
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=DEV)
        out = torch.full(q.shape, 7.0, dtype=torch.float16, device=DEV)

        def call():
            K.tq_attention_paged(q, c["kp"], c["kn"], c["vp"], c["vn"], torch.from_numpy(c["tables"]).to(DEV),
                                 torch.tensor(kv_lens, dtype=torch.int32, device=DEV),
                                 torch.tensor(starts, dtype=torch.int32, device=DEV), c["pik"], c["piv"], c["ck"],
                                 c["cv"], kb, vb, out, max_kv_len=L, workspace=ws)
            torch.cuda.synchronize()

        _, served = _run_counted("attention_streamed", call)
        assert served == 1
        got = out.float().cpu().numpy()
        for s, Ls in enumerate(kv_lens):
            ops.assert_close_fp(got[s], statement(c, qh[s], s, Ls, starts[s]), rel=2e-3, min_cos=0.9999,
                                label=f"ws {ws_bytes} seq {s} (kv {Ls})", dtype="f16")
