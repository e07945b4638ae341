"""GPU parity of the elementwise kernels against the CPU oracle (and the fixture goldens).

Tolerances: the north-star bar for FP16/BF16 outputs — max-abs error within
2e-3 of the reference magnitude, beyond the output dtype's own rounding (half
an ulp, which for BF16 alone can reach 3.9e-3 of a value), and cosine >= 0.9999
against a float64 computation (``oracle.ops.assert_close_fp``); bit-exact for the embedding
gather and for the residual add's stored sum. The fixture tests additionally
apply the reference harness's own rule ``|a-e| <= atol + rtol*|e|``
(tests/model-validation/tests/kernels.rs:118-123, :1551-1552).
"""

import numpy as np
import pytest
import torch

from fracture_b200 import kernels as K
from oracle import ops

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
TDT = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}


def to_dev(x, dt):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(DEV).to(TDT[dt])


def to_np(t):
    return t.detach().float().cpu().numpy()


def rand(shape, seed, scale=1.0, outliers=0.0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(shape).astype(np.float32) * scale
    if outliers:
        x[..., rng.random(shape[-1]) < outliers] *= 20.0
    return x


# ── silu_mul / add ───────────────────────────────────────────────────────────

@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("n", [1, 7, 8, 1000, 4096 * 3 + 5, 64 * 14336])
def test_silu_mul(dt, n):
    g = ops.round_to(rand((n,), 1, 3.0), dt)
    u = ops.round_to(rand((n,), 2), dt)
    out = torch.empty(n, dtype=TDT[dt], device=DEV)
    K.silu_mul(out, to_dev(g, dt), to_dev(u, dt))
    torch.cuda.synchronize()
    ops.assert_close_fp(to_np(out), ops.silu_mul(g, u, "f32"), label=f"silu {dt} {n}", dtype=dt)


def test_silu_mul_unaligned_and_extremes():
    dt = "f16"
    g = np.array([-100.0, -20.0, -1.0, 0.0, 1.0, 20.0, 60000.0, -60000.0, 3.0], dtype=np.float32)
    u = np.ones_like(g)
    big_g = torch.zeros(g.size + 1, dtype=torch.float16, device=DEV)
    big_u = torch.zeros(g.size + 1, dtype=torch.float16, device=DEV)
    big_o = torch.zeros(g.size + 1, dtype=torch.float16, device=DEV)
    big_g[1:] = to_dev(g, dt)
    big_u[1:] = to_dev(u, dt)
    K.silu_mul(big_o[1:], big_g[1:], big_u[1:])  # 2-byte offset: not 16-byte aligned
    torch.cuda.synchronize()
    got = to_np(big_o[1:])
    ref = ops.silu_mul(ops.round_to(g, dt), u, dt)
    assert np.all(np.isfinite(got[:6])) and np.allclose(got, ref, rtol=2e-3, atol=1e-6)


@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("n", [3, 4096, 32768 + 3])
def test_add_bit_exact_and_in_place(dt, n):
    a = ops.round_to(rand((n,), 3, 100.0), dt)
    b = ops.round_to(rand((n,), 4), dt)
    ta, tb = to_dev(a, dt), to_dev(b, dt)
    out = torch.empty_like(ta)
    K.add(out, ta, tb)
    K.add(ta, ta, tb)  # in place, as the engine calls it
    torch.cuda.synchronize()
    ref = ops.add(a, b, dt)
    assert np.array_equal(to_np(out), ref) and np.array_equal(to_np(ta), ref)


# ── embedding ────────────────────────────────────────────────────────────────

@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("vocab,hidden,ntok", [(256, 64, 32), (256, 128, 24), (1000, 4096, 64), (50, 12, 9)])
def test_embedding_bit_exact_with_oov(dt, vocab, hidden, ntok):
    table = ops.round_to(rand((vocab, hidden), 5, 0.02), dt)
    ids = np.random.default_rng(6).integers(0, vocab, ntok).astype(np.uint32)
    ids[::5] = vocab + 3  # out of vocabulary -> zero row (embedding.cu:21-25)
    ids[-1] = 0xFFFFFFFF
    out = torch.full((ntok, hidden), 7.0, dtype=TDT[dt], device=DEV)
    K.embedding(out, to_dev(table, dt), torch.from_numpy(ids.view(np.int32)).to(DEV))
    torch.cuda.synchronize()
    assert np.array_equal(to_np(out), ops.embedding(table, ids))


# ── rmsnorm / add+rmsnorm ────────────────────────────────────────────────────

@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("rows,cols", [(32, 64), (24, 128), (64, 4096), (3, 8192), (5, 100), (2, 16384 + 8)])
def test_rmsnorm(dt, rows, cols):
    x = ops.round_to(rand((rows, cols), 7, 2.0, outliers=0.001), dt)
    w = ops.round_to(1.0 + rand((cols,), 8, 0.02), dt)
    out = torch.empty((rows, cols), dtype=TDT[dt], device=DEV)
    K.rmsnorm(out, to_dev(x, dt), to_dev(w, dt), 1e-5)
    torch.cuda.synchronize()
    ops.assert_close_fp(to_np(out), ops.rmsnorm(x, w, 1e-5, "f32"), label=f"rmsnorm {dt} {rows}x{cols}", dtype=dt)


@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("rows,cols", [(32, 64), (64, 4096), (7, 8192), (4, 136)])
def test_add_rmsnorm_fused(dt, rows, cols):
    h = ops.round_to(rand((rows, cols), 9, 5.0, outliers=0.001), dt)
    r = ops.round_to(rand((rows, cols), 10), dt)
    w = ops.round_to(1.0 + rand((cols,), 11, 0.02), dt)
    th = to_dev(h, dt)
    normed = torch.empty_like(th)
    K.add_rmsnorm(th, to_dev(r, dt), to_dev(w, dt), normed, 1e-5)
    torch.cuda.synchronize()
    h_ref, _ = ops.add_rmsnorm(h, r, w, 1e-5, dt)
    assert np.array_equal(to_np(th), h_ref)  # the stored residual is bit-exact
    ops.assert_close_fp(to_np(normed), ops.rmsnorm(h_ref, w, 1e-5, "f32"), label=f"add_rmsnorm {dt}", dtype=dt)


def test_rmsnorm_zero_rows():
    x = np.zeros((4, 4096), np.float32)
    out = torch.full((4, 4096), 3.0, dtype=torch.float16, device=DEV)
    K.rmsnorm(out, to_dev(x, "f16"), to_dev(np.ones(4096), "f16"), 1e-5)
    torch.cuda.synchronize()
    assert not to_np(out).any()


# ── rope ─────────────────────────────────────────────────────────────────────

@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
@pytest.mark.parametrize("T,nq,nkv,hd,maxpos,llama3", [
    (32, 4, 2, 16, 32, False),        # BASELINE config 1 shapes
    (24, 4, 2, 32, 24, False),        # fixture shapes
    (64, 32, 8, 128, 8192, True),     # config 2: decode, positions up to 8191, llama3
    (300, 32, 8, 128, 2048, True),    # prefill-like
    (5, 3, 1, 6, 100, False),         # scalar path: head_dim/2 not a multiple of the vector width
])
def test_rope(dt, T, nq, nkv, hd, maxpos, llama3):
    rng = np.random.default_rng(12)
    q = ops.round_to(rand((T, nq, hd), 13), dt)
    k = ops.round_to(rand((T, nkv, hd), 14), dt)
    pos = rng.integers(0, maxpos, T).astype(np.uint32) if maxpos > T else np.arange(T, dtype=np.uint32)
    f = (K.rope_freqs_llama3(hd, 5e5, 8.0, 1.0, 4.0, 8192) if llama3 else K.rope_freqs(hd, 5e5))
    tq_, tk = to_dev(q, dt), to_dev(k, dt)
    K.rope(tq_, tk, torch.from_numpy(pos.view(np.int32)).to(DEV), torch.from_numpy(f).to(DEV))
    torch.cuda.synchronize()
    ops.assert_close_fp(to_np(tq_), ops.rope(q, pos, f, "f32"), label="rope q", dtype=dt)
    ops.assert_close_fp(to_np(tk), ops.rope(k, pos, f, "f32"), label="rope k", dtype=dt)


# ── reference fixture goldens through the raw kernels ───────────────────────

@pytest.mark.parametrize("p", [0, 1])
def test_fixture_layers(golden, p):
    z = golden[p]
    import json

    m = json.loads(bytes(z["meta_json"]))
    eps, hd = m["rms_norm_eps"], m["head_dim"]
    f = torch.from_numpy(K.rope_freqs(hd, m["rope_theta"])).to(DEV)
    if "embeddings" in z.files:
        ids = torch.from_numpy(z["token_ids"]).to(DEV)
        tab = to_dev(z["token_embd"].astype(np.float32), "f16")
        out = torch.empty((ids.numel(), tab.shape[1]), dtype=torch.float16, device=DEV)
        K.embedding(out, tab, ids)
        torch.cuda.synchronize()
        assert np.array_equal(to_np(out), z["embeddings"])
    for l in range(m["num_layers"]):
        x = to_dev(z[f"l{l}.input_hidden"], "f16")
        w = to_dev(z[f"l{l}.attn_norm_w"].astype(np.float32), "f16")
        out = torch.empty_like(x)
        K.rmsnorm(out, x, w, eps)
        torch.cuda.synchronize()
        assert ops.compare_tensors(to_np(out), z[f"l{l}.post_attn_norm"], 5e-3, 5e-3) == 0
        # fused residual add + ffn norm; the add is pinned bit-exactly by output_hidden
        h = to_dev(z[f"l{l}.post_attn_residual"], "f16")
        wf = to_dev(z[f"l{l}.ffn_norm_w"].astype(np.float32), "f16")
        normed = torch.empty_like(h)
        K.rmsnorm(normed, h, wf, eps)
        torch.cuda.synchronize()
        assert ops.compare_tensors(to_np(normed), z[f"l{l}.post_ffn_norm"], 5e-3, 5e-3) == 0
        K.add_rmsnorm(h, to_dev(z[f"l{l}.ffn_output"], "f16"), wf, normed, eps)
        torch.cuda.synchronize()
        assert np.array_equal(to_np(h), z[f"l{l}.output_hidden"])
        T = z[f"l{l}.q"].shape[0]
        q = to_dev(z[f"l{l}.q"], "f16").view(T, m["num_q_heads"], hd)
        k = to_dev(z[f"l{l}.k"], "f16").view(T, m["num_kv_heads"], hd)
        K.rope(q, k, torch.arange(T, dtype=torch.int32, device=DEV), f)
        torch.cuda.synchronize()
        assert ops.compare_tensors(to_np(q), z[f"l{l}.q_rope"], 0.01, 0.025) == 0
        assert ops.compare_tensors(to_np(k), z[f"l{l}.k_rope"], 0.01, 0.025) == 0
        if f"l{l}.silu_mul" in z.files:
            g, u = to_dev(z[f"l{l}.gate"], "f16"), to_dev(z[f"l{l}.up"], "f16")
            o = torch.empty_like(g)
            K.silu_mul(o, g, u)
            torch.cuda.synchronize()
            assert ops.compare_tensors(to_np(o), z[f"l{l}.silu_mul"], 1e-3, 1e-3) == 0


# ── full-size properties (config 3 shapes) ──────────────────────────────────

def test_prefill_sized_chain_properties():
    """At 16x2048 tokens: h += r is exact (checked on a sample of rows), rope preserves
    norms per head to fp rounding, silu_mul is odd-symmetric in (g, u) -> (g, -u)."""
    T, H, I = 32768, 4096, 14336
    g = torch.Generator(device=DEV).manual_seed(0)
    h = torch.randn((T, H), generator=g, device=DEV).to(torch.bfloat16)
    r = torch.randn((T, H), generator=g, device=DEV).to(torch.bfloat16)
    w = torch.ones(H, device=DEV, dtype=torch.bfloat16)
    h0 = h.clone()
    normed = torch.empty_like(h)
    K.add_rmsnorm(h, r, w, normed, 1e-5)
    rows = torch.arange(0, T, 997, device=DEV)
    ref = (h0[rows].float() + r[rows].float()).to(torch.bfloat16)
    assert torch.equal(h[rows], ref)
    rms = normed[rows].float().pow(2).mean(-1).sqrt()
    assert torch.allclose(rms, torch.ones_like(rms), atol=1e-2)
    q = torch.randn((T, 32, 128), generator=g, device=DEV).to(torch.bfloat16)
    n0 = q.float().norm(dim=-1)
    k = torch.randn((T, 8, 128), generator=g, device=DEV).to(torch.bfloat16)
    pos = (torch.arange(T, device=DEV) % 2048).to(torch.int32)
    K.rope(q, k, pos, torch.from_numpy(K.rope_freqs_llama3(128, 5e5, 8, 1, 4, 8192)).to(DEV))
    assert torch.allclose(q.float().norm(dim=-1), n0, rtol=1e-2)
    del q, k, h, r, normed
    gt = torch.randn((4096, I), generator=g, device=DEV).to(torch.bfloat16)
    up = torch.randn((4096, I), generator=g, device=DEV).to(torch.bfloat16)
    o1, o2 = torch.empty_like(gt), torch.empty_like(gt)
    K.silu_mul(o1, gt, up)
    K.silu_mul(o2, gt, -up)
    torch.cuda.synchronize()
    assert torch.equal(o1, -o2)


def test_config3_chain_sampled_rows_meet_the_bar():
    """The headline workload's inputs (bench.py config 3): 16 x 2048 BF16 tokens, hidden 4096,
    32/8 heads of 128, intermediate 14336, the full 128,256-row embedding table, N(0,1)
    activations with 0.1% of the channels x20, llama3 RoPE at positions 0..2047 per sequence.
    Two layers of the chain run over all 32768 tokens; 384 sampled rows of every output are
    held to the north-star bar (max-abs 2e-3 of magnitude beyond BF16 rounding, cosine >= 0.9999)
    against the float64 oracle, and the residual stream h stays bit-exact."""
    T, HID, NQ, NKV, HD, INTER, VOCAB, EPS = 32768, 4096, 32, 8, 128, 14336, 128256, 1e-5
    bf = torch.bfloat16
    g = torch.Generator(device=DEV).manual_seed(1234)

    def act(shape):
        x = torch.randn(shape, generator=g, device=DEV)
        cols = torch.rand(shape[-1], generator=g, device=DEV) < 0.001
        return torch.where(cols, x * 20.0, x).to(bf)

    table = (torch.randn((VOCAB, HID), generator=g, device=DEV) * 0.02).to(bf)
    ids = torch.randint(0, VOCAB, (T,), generator=g, device=DEV, dtype=torch.int32)
    pos = (torch.arange(T, device=DEV, dtype=torch.int32) % 2048).contiguous()
    attn_proj, ffn_out = act((T, HID)), act((T, HID))
    q, k = act((T, NQ, HD)), act((T, NKV, HD))
    gate, up = act((T, INTER)), act((T, INTER))
    wa = (1 + 0.02 * torch.randn((2, HID), generator=g, device=DEV)).to(bf)
    wf = (1 + 0.02 * torch.randn((2, HID), generator=g, device=DEV)).to(bf)
    freqs = K.rope_freqs_llama3(HD, 5e5, 8.0, 1.0, 4.0, 8192)
    rows = torch.from_numpy(np.sort(np.random.default_rng(3).choice(T, 384, replace=False))).to(DEV)
    rnp = rows.cpu().numpy()
    host = lambda t: t[rows].float().cpu().numpy()
    h = torch.empty((T, HID), device=DEV, dtype=bf)
    normed = torch.empty_like(h)
    mid = torch.empty_like(gate)
    q0, k0 = host(q), host(k)

    K.embedding(h, table, ids)
    torch.cuda.synchronize()
    h_ref = ops.embedding(table[ids[rows].long()].float().cpu().numpy(), np.arange(len(rnp)))
    assert np.array_equal(host(h), h_ref)
    a_ref, f_ref = host(attn_proj), host(ffn_out)
    gt, ut = host(gate), host(up)
    for l in range(2):
        wa_h, wf_h = wa[l].float().cpu().numpy(), wf[l].float().cpu().numpy()
        if l == 0:
            K.rmsnorm(normed, h, wa[0], EPS)
            n_ref = ops.rmsnorm(h_ref, wa_h, EPS, "f32")
        else:
            K.add_rmsnorm(h, ffn_out, wa[l], normed, EPS)
            h_ref = ops.add(h_ref, f_ref, "bf16")
            n_ref = ops.rmsnorm(h_ref, wa_h, EPS, "f32")
        torch.cuda.synchronize()
        assert np.array_equal(host(h), h_ref), f"layer {l}: residual stream"
        ops.assert_close_fp(host(normed), n_ref, label=f"layer {l} attn norm", dtype="bf16")
        K.rope(q, k, pos, torch.from_numpy(freqs).to(DEV))
        torch.cuda.synchronize()
        q0 = ops.round_to(ops.rope(q0, rnp % 2048, freqs, "f32"), "f32")
        k0 = ops.round_to(ops.rope(k0, rnp % 2048, freqs, "f32"), "f32")
        ops.assert_close_fp(host(q), q0, label=f"layer {l} rope q", dtype="bf16")
        ops.assert_close_fp(host(k), k0, label=f"layer {l} rope k", dtype="bf16")
        q0, k0 = host(q), host(k)  # the next layer rotates the stored BF16 values again
        K.add_rmsnorm(h, attn_proj, wf[l], normed, EPS)
        h_ref = ops.add(h_ref, a_ref, "bf16")
        torch.cuda.synchronize()
        assert np.array_equal(host(h), h_ref), f"layer {l}: residual stream after attention"
        ops.assert_close_fp(host(normed), ops.rmsnorm(h_ref, wf_h, EPS, "f32"), label=f"layer {l} ffn norm",
                            dtype="bf16")
        K.silu_mul(mid, gate, up)
        torch.cuda.synchronize()
        ops.assert_close_fp(host(mid), ops.silu_mul(gt, ut, "f32"), label=f"layer {l} silu_mul", dtype="bf16")
