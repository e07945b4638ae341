"""The float64 statement of the reference's paged attention kernel (``oracle.ops.attention_paged``,
``backends/fracture-cuda/kernels/attention_paged.cu:25-155``) against torch's
``scaled_dot_product_attention`` in float64 on the CPU, over the same keys and values laid out
contiguously: shuffled block tables, GQA groups, causal prefill offsets, a missing block and an
empty context. (The GPU tests pin the statement to the reference kernel itself.)"""

import numpy as np
import pytest
import torch

from oracle import ops

D = 128


def _paged(k, v, rng):
    """Scatter contiguous k, v [L, Hkv, D] into pools through a shuffled block table."""
    L, Hkv, _ = k.shape
    nb = (L + 15) // 16
    total = nb + 3
    table = rng.permutation(total)[:nb].astype(np.int64)
    kp = np.full((total * 16, Hkv, D), 1e3)
    vp = np.full((total * 16, Hkv, D), 1e3)
    pos = np.arange(L)
    rows = table[pos // 16] * 16 + pos % 16
    kp[rows], vp[rows] = k, v
    return kp, vp, table


def _sdpa(q, k, v, start, kv_len, keep=None):
    """torch SDPA, float64: query t sees positions [0, min(start + t + 1, kv_len)) (and keep)."""
    N, Hq, _ = q.shape
    G = Hq // k.shape[1]
    kk = torch.from_numpy(np.repeat(k[:kv_len], G, axis=1)).permute(1, 0, 2)  # [Hq, L, D]
    vv = torch.from_numpy(np.repeat(v[:kv_len], G, axis=1)).permute(1, 0, 2)
    qq = torch.from_numpy(q).permute(1, 0, 2)                                  # [Hq, N, D]
    mask = np.arange(kv_len)[None, :] < np.minimum(start + np.arange(N) + 1, kv_len)[:, None]
    if keep is not None:
        mask &= keep[None, :kv_len]
    out = torch.nn.functional.scaled_dot_product_attention(qq, kk, vv, attn_mask=torch.from_numpy(mask))
    out = out.permute(1, 0, 2).numpy()
    out[~mask.any(1)] = 0.0
    return out


@pytest.mark.parametrize("L,N,Hq,Hkv", [(1, 1, 4, 1), (37, 1, 8, 2), (300, 5, 8, 8), (513, 9, 16, 2)])
def test_statement_equals_sdpa(L, N, Hq, Hkv):
    rng = np.random.default_rng(L + N)
    k = rng.standard_normal((L, Hkv, D)) * 1.5
    v = rng.standard_normal((L, Hkv, D))
    q = rng.standard_normal((N, Hq, D))
    kp, vp, table = _paged(k, v, rng)
    start = L - N
    got = ops.attention_paged(q, kp, vp, table, L, start)
    np.testing.assert_allclose(got, _sdpa(q, k, v, start, L), rtol=1e-10, atol=1e-12)


def test_missing_block_and_empty_context():
    rng = np.random.default_rng(5)
    L, Hkv, Hq = 70, 2, 4
    k = rng.standard_normal((L, Hkv, D))
    v = rng.standard_normal((L, Hkv, D))
    q = rng.standard_normal((2, Hq, D))
    kp, vp, table = _paged(k, v, rng)
    table[1] = -1  # positions 16..31 left out
    keep = np.ones(L, bool)
    keep[16:32] = False
    got = ops.attention_paged(q, kp, vp, table, L, L - 2)
    np.testing.assert_allclose(got, _sdpa(q, k, v, L - 2, L, keep), rtol=1e-10, atol=1e-12)
    assert not np.any(ops.attention_paged(q, kp, vp, table, 0, 0))
