"""launch_attention_paged_tq_noalloc against launch_attention_paged_tq, through the C ABI.

Who needs this entry point: an engine that sized its TurboQuant KV pool to take all free device
memory at start-up cannot have a cudaMalloc succeed in the middle of a step, and a decode loop
cannot afford the device-wide synchronisation of the cudaFree that growing the library workspace
of launch_attention_paged_tq implies. The no-allocation variant keeps its rotated queries and
split-K partials in one fixed 4 MiB device array inside the library instead.

Both entry points run the same kernels, so their outputs must agree bit for bit (stricter than
the 2e-3 / cosine 0.9999 bar the attention tests use against the float64 statement, which the
no-allocation output is also held to here). Two calls in a row with different shapes check that
what the shared array keeps from the previous call never leaks into the next one. The file sorts
last so that it also runs after every other GPU test in one process, and it builds all of its
own data so that it also passes alone in a fresh process.
"""

import numpy as np
import pytest
import torch

from fracture_b200 import _lib
from fracture_b200 import kernels as K
from oracle import ops, turboquant as tq

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
D = 128
SCRATCH = 4 << 20  # FB_TQA_NOALLOC_SCRATCH_BYTES


def need_bytes(num_tokens, num_q_heads, kv_len):
    """Scratch a call takes: rotated queries plus one partial per 256-position chunk and head."""
    return num_tokens * num_q_heads * (D * 4 + (D + 2) * 4 * ((kv_len + 255) // 256))


def build_cache(kv_len, Hkv, kb, vb, seed):
    """One sequence of kv_len positions in shuffled 16-row blocks, written by the compress kernels."""
    rng = np.random.default_rng(seed)
    nblk = (kv_len + 15) // 16
    total = nblk + 3
    table = rng.permutation(total)[:nblk].astype(np.int32)
    rows = total * 16
    Pk, Pv = D * kb // 8, D * vb // 8
    c = {"kp": torch.zeros((rows, Hkv * Pk), dtype=torch.uint8, device=DEV),
         "vp": torch.zeros((rows, Hkv * Pv), dtype=torch.uint8, device=DEV),
         "kn": torch.zeros((rows, Hkv), dtype=torch.float16, device=DEV),
         "vn": torch.zeros((rows, Hkv), dtype=torch.float16, device=DEV)}
    host = {"pik": K.tq_rotation_matrix(D, seed), "piv": K.tq_rotation_matrix(D, seed + 500),
            "ck": K.tq_codebook(D, kb)[0], "cv": K.tq_codebook(D, vb)[0]}
    for n, x in host.items():
        c[n] = torch.from_numpy(np.ascontiguousarray(x)).to(DEV)
    bt = torch.from_numpy(table).to(DEV)
    kx = torch.from_numpy((rng.standard_normal((kv_len, Hkv, D)) * 1.5).astype(np.float32)).to(DEV).half()
    vx = torch.from_numpy(rng.standard_normal((kv_len, Hkv, D)).astype(np.float32)).to(DEV).half()
    K.tq_compress_paged(kx, c["pik"], c["ck"], kb, c["kp"], c["kn"], block_table=bt)
    K.tq_compress_paged(vx, c["piv"], c["cv"], vb, c["vp"], c["vn"], block_table=bt)
    arr = lambda base, stride: torch.tensor([base + b * 16 * stride for b in range(total)], dtype=torch.int64,
                                            device=DEV)
    c["ptrs"] = (arr(c["kp"].data_ptr(), Hkv * Pk), arr(c["kn"].data_ptr(), Hkv * 2),
                 arr(c["vp"].data_ptr(), Hkv * Pv), arr(c["vn"].data_ptr(), Hkv * 2))
    c.update(table=table, bt=bt, kb=kb, vb=vb, Hkv=Hkv, kv_len=kv_len, host=host)
    torch.cuda.synchronize()
    return c


def call(fn_name, c, q, start):
    """One call of the named reference-ABI entry point; returns the FP16 output."""
    Tq, Hq, _ = q.shape
    kp, kn, vp, vn = c["ptrs"]
    out = torch.full((Tq, Hq, D), 7.0, dtype=torch.float16, device=DEV)
    rc = getattr(_lib.load(), fn_name)(
        out.data_ptr(), q.data_ptr(), c["bt"].data_ptr(), kp.data_ptr(), kn.data_ptr(), vp.data_ptr(), vn.data_ptr(),
        c["pik"].data_ptr(), c["piv"].data_ptr(), c["ck"].data_ptr(), c["cv"].data_ptr(), Tq, Hq, c["Hkv"], D,
        c["kv_len"], start, c["kb"], c["vb"], D * c["kb"] // 8, D * c["vb"] // 8,
        torch.cuda.current_stream().cuda_stream)
    assert rc == 0, (fn_name, rc, _lib.load().fb_last_error())
    return out


def make_q(Tq, Hq, seed):
    x = ops.round_to(np.random.default_rng(seed).standard_normal((Tq, Hq, D)).astype(np.float32), "f16")
    return x, torch.from_numpy(x).to(DEV).half()


def statement(c, qh, start):
    h = c["host"]
    return tq.attention_paged_tq(qh, c["kp"].cpu().numpy(), c["kn"].float().cpu().numpy(), c["vp"].cpu().numpy(),
                                 c["vn"].float().cpu().numpy(), c["table"], c["kv_len"], start, h["pik"], h["piv"],
                                 h["ck"], h["cv"], c["kb"], c["vb"], c["Hkv"])


def test_noalloc_equals_allocating_entry_on_two_calls_in_a_row():
    """A 7-token prefill chunk over 2100 positions (tensor-core path, 4/2-bit), then one decode token
    over 900 positions with 8-bit codes (CUDA-core path): each equals launch_attention_paged_tq bit
    for bit and meets the FP bar against the float64 statement."""
    cases = [(2100, 2, 4, 4, 2, 7), (900, 2, 8, 8, 8, 1)]  # kv_len, Hkv, G, kb, vb, query tokens
    for i, (kv_len, Hkv, G, kb, vb, Tq) in enumerate(cases):
        c = build_cache(kv_len, Hkv, kb, vb, seed=30 + i)
        qh, q = make_q(Tq, G * Hkv, seed=40 + i)
        start = kv_len - Tq
        ref = call("launch_attention_paged_tq", c, q, start)
        got = call("launch_attention_paged_tq_noalloc", c, q, start)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"call {i}: outputs differ"
        ops.assert_close_fp(got.float().cpu().numpy(), statement(c, qh, start), rel=2e-3, min_cos=0.9999,
                            label=f"call {i}", dtype="f16")


def test_noalloc_at_its_limit_allocates_nothing():
    """One decode token with 32 Q heads at the longest context the scratch holds: after the first
    call (which loads the module and looks the array's address up), further calls leave free device
    memory unchanged and keep matching the allocating entry point."""
    Hkv, G = 8, 4
    kv_len = 256 * ((SCRATCH // (G * Hkv) - D * 4) // ((D + 2) * 4))
    assert need_bytes(1, G * Hkv, kv_len) <= SCRATCH < need_bytes(1, G * Hkv, kv_len + 256)
    c = build_cache(kv_len, Hkv, 4, 2, seed=50)
    qs = [make_q(1, G * Hkv, seed=51 + i)[1] for i in range(2)]
    call("launch_attention_paged_tq_noalloc", c, qs[0], kv_len - 1)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    got = [call("launch_attention_paged_tq_noalloc", c, q, kv_len - 1) for q in qs]
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    # the outputs above come from torch's caching allocator; nothing else may take device memory
    assert free1 >= free0 - (2 << 20), (free0, free1)
    for q, g in zip(qs, got):
        assert torch.equal(g, call("launch_attention_paged_tq", c, q, kv_len - 1))


def test_noalloc_rejects_a_call_beyond_its_scratch():
    """A call needing more than the fixed array is refused with the reason, before any launch."""
    lib = _lib.load()
    Hkv, G = 8, 4
    kv_len = 256 * ((SCRATCH // (G * Hkv) - D * 4) // ((D + 2) * 4)) + 256
    assert need_bytes(1, G * Hkv, kv_len) > SCRATCH
    dummy = torch.zeros(64, dtype=torch.int64, device=DEV)
    p = dummy.data_ptr()
    rc = lib.launch_attention_paged_tq_noalloc(p, p, p, p, p, p, p, p, p, p, p, 1, G * Hkv, Hkv, D, kv_len,
                                               kv_len - 1, 4, 2, D // 2, D // 4, torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    msg = lib.fb_last_error().decode()
    assert "launch_attention_paged_tq_noalloc" in msg and str(SCRATCH) in msg
    torch.cuda.synchronize()
