"""Both paged attention paths at the bench's decode size (64 sequences x 1 query token at the end
of an 8192-token context, 32 Q / 8 KV heads x 128, shuffled block tables over one pool), and at
4 and 1 sequences (the tensor-core kernels pick 2048-, 1024- and 512-position items), through
a size-independent identity instead of the float64 statement (which would take minutes here):

* TurboQuant cache: the attention equals plain softmax attention over the cache as this
  library's dequantize reconstructs it (scores in K's rotated space are q . x_hat / sqrt(d),
  and the value sum rotated back is the sum of the reconstructed values);
* FP16 cache: the attention equals plain softmax attention over the rows the block table
  addresses.

References: torch scaled_dot_product_attention in float32 on the GPU. Bar as in the other
attention tests (max-abs 2e-3 of the magnitude beyond FP16 rounding, cosine >= 0.9999).
"""

import numpy as np
import pytest
import torch

from fracture_b200 import kernels as K
from oracle import ops

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
L, HQ, HKV, D = 8192, 32, 8, 128
NB = L // 16
BATCHES = [64, 4, 1]


def _setup(seed, S):
    g = torch.Generator(device=DEV).manual_seed(seed)
    tables = torch.randperm(S * NB, generator=g, device=DEV).to(torch.int32).view(S, NB)
    q = torch.randn((S, 1, HQ, D), generator=g, device=DEV).half()
    kv_lens = torch.full((S,), L, dtype=torch.int32, device=DEV)
    starts = torch.full((S,), L - 1, dtype=torch.int32, device=DEV)
    return g, tables, q, kv_lens, starts


def _sdpa(q, k, v):
    """q [1, HQ, D], k/v [L, HKV, D] (any float dtype) -> [1, HQ, D] float32."""
    kk = k.float().repeat_interleave(HQ // HKV, dim=1).permute(1, 0, 2)
    vv = v.float().repeat_interleave(HQ // HKV, dim=1).permute(1, 0, 2)
    out = torch.nn.functional.scaled_dot_product_attention(q.float().permute(1, 0, 2), kk, vv)
    return out.permute(1, 0, 2)


@pytest.mark.parametrize("S", BATCHES)
def test_tq_attention_equals_attention_over_the_dequantized_cache(S):
    g, tables, q, kv_lens, starts = _setup(21, S)
    KB, VB = 4, 2
    rows = S * L
    kp = torch.empty((rows, HKV * D * KB // 8), dtype=torch.uint8, device=DEV)
    vp = torch.empty((rows, HKV * D * VB // 8), dtype=torch.uint8, device=DEV)
    kn = torch.empty((rows, HKV), dtype=torch.float16, device=DEV)
    vn = torch.empty((rows, HKV), dtype=torch.float16, device=DEV)
    pik, piv = (torch.from_numpy(K.tq_rotation_matrix(D, sd)).to(DEV) for sd in (42, 542))
    ck, cv = (torch.from_numpy(K.tq_codebook(D, b)[0]).to(DEV) for b in (KB, VB))
    for s in range(S):
        K.tq_compress_paged(torch.randn((L, HKV, D), generator=g, device=DEV).half() * 1.5, pik, ck, KB, kp, kn,
                            block_table=tables[s])
        K.tq_compress_paged(torch.randn((L, HKV, D), generator=g, device=DEV).half(), piv, cv, VB, vp, vn,
                            block_table=tables[s])
    out = torch.empty_like(q)
    K.tq_attention_paged(q, kp, kn, vp, vn, tables, kv_lens, starts, pik, piv, ck, cv, KB, VB, out, max_kv_len=L)
    khat = torch.empty((L, HKV, D), dtype=torch.float16, device=DEV)
    vhat = torch.empty_like(khat)
    ref = torch.empty((S, HQ, D), dtype=torch.float32, device=DEV)
    for s in range(S):
        K.tq_dequant_paged(kp, kn, pik, ck, KB, khat, block_table=tables[s])
        K.tq_dequant_paged(vp, vn, piv, cv, VB, vhat, block_table=tables[s])
        ref[s] = _sdpa(q[s], khat, vhat)[0]
    torch.cuda.synchronize()
    ops.assert_close_fp(out[:, 0].float().cpu().numpy(), ref.cpu().numpy(), rel=2e-3, min_cos=0.9999,
                        label=f"TurboQuant attention, {S} x 8192", dtype="f16")


@pytest.mark.parametrize("S", BATCHES)
def test_fp16_attention_equals_attention_over_the_addressed_rows(S):
    g, tables, q, kv_lens, starts = _setup(22, S)
    kpool = torch.empty((S * L, HKV, D), dtype=torch.float16, device=DEV)
    vpool = torch.empty_like(kpool)
    for s in range(S):
        K.kv_append_paged(torch.randn((L, HKV, D), generator=g, device=DEV).half() * 1.5,
                          torch.randn((L, HKV, D), generator=g, device=DEV).half(), kpool, vpool, tables[s])
    out = torch.empty_like(q)
    K.attention_paged(q, kpool, vpool, tables, kv_lens, starts, out, max_kv_len=L)
    pos = torch.arange(L, device=DEV)
    ref = torch.empty((S, HQ, D), dtype=torch.float32, device=DEV)
    for s in range(S):
        rows = tables[s][pos // 16].long() * 16 + pos % 16
        ref[s] = _sdpa(q[s], kpool[rows], vpool[rows])[0]
    torch.cuda.synchronize()
    ops.assert_close_fp(out[:, 0].float().cpu().numpy(), ref.cpu().numpy(), rel=2e-3, min_cos=0.9999,
                        label=f"FP16 attention, {S} x 8192", dtype="f16")
