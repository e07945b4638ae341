"""The reference's CPU numerical path for the per-layer elementwise chain (timed baseline).

Test infrastructure only: ``bench.py`` times it as the CPU baseline (its
``cpu_baseline`` leg and its ``--impl reference`` arm); nothing in the product
calls it.

It is the PyTorch math the reference's validation scripts use on the host,
run with torch on the CPU with every available thread:

* RoPE — ``scripts/dump_reference.py:274-286`` (f32 angle = position * inv_freq,
  cos/sin, split-half rotation ``x*cos + rotate_half(x)*sin`` in float32,
  ``:307-323``);
* SiLU·mul — ``silu(gate) * up`` (``dump_reference.py:243-250``) in float32;
* RMSNorm and the residual add — the kernel formulas (``kernels/rmsnorm.cu:24-66``,
  ``kernels/add.cu:13``) in float32 with one final rounding;
* embedding — an index select with zero rows for out-of-vocabulary ids.

Storage is the activation dtype (BF16 for BASELINE config 3); math is float32.
"""

from __future__ import annotations

import os
import time

import torch


def set_threads() -> int:
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    torch.set_num_threads(n)
    return n


def embedding(ids: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    vocab = table.shape[0]
    ok = ids < vocab
    out = table.index_select(0, torch.where(ok, ids, torch.zeros_like(ids)))
    return torch.where(ok[:, None], out, torch.zeros((), dtype=table.dtype))


def add_rmsnorm(h: torch.Tensor, r: torch.Tensor | None, w: torch.Tensor, eps: float):
    if r is not None:
        h = (h.float() + r.float()).to(h.dtype)
    x = h.float()
    inv = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return h, (x * inv * w.float()).to(h.dtype)


def rope(x: torch.Tensor, positions: torch.Tensor, inv_freq: torch.Tensor) -> torch.Tensor:
    ang = positions.to(torch.float32)[:, None] * inv_freq[None, :]
    ang = torch.cat((ang, ang), dim=-1)
    cos, sin = ang.cos()[:, None, :], ang.sin()[:, None, :]
    x32 = x.float()
    half = x32.shape[-1] // 2
    rot = torch.cat((-x32[..., half:], x32[..., :half]), dim=-1)
    return (x32 * cos + rot * sin).to(x.dtype)


def silu_mul(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    return (torch.nn.functional.silu(g.float()) * u.float()).to(g.dtype)


def layer_chain(h, attn_out, ffn_out, q, k, gate, up, wa, wf, positions, inv_freq, eps, first: bool):
    """One layer of the elementwise chain as the engine orders it (batched.rs:290-402)."""
    h, normed = add_rmsnorm(h, None if first else ffn_out, wa, eps)
    q = rope(q, positions, inv_freq)
    k = rope(k, positions, inv_freq)
    h, normed = add_rmsnorm(h, attn_out, wf, eps)
    mid = silu_mul(gate, up)
    return h, normed, q, k, mid


def make_data(tokens: int, hidden: int, nq: int, nkv: int, head_dim: int, inter: int, layers: int, vocab: int,
              dtype=torch.bfloat16, seed: int = 0) -> dict:
    g = torch.Generator().manual_seed(seed)
    return {
        "table": (torch.randn((vocab, hidden), generator=g) * 0.02).to(dtype),
        "ids": torch.randint(0, vocab, (tokens,), generator=g),
        "positions": torch.arange(tokens) % 2048,
        "attn_out": torch.randn((tokens, hidden), generator=g).to(dtype),
        "ffn_out": torch.randn((tokens, hidden), generator=g).to(dtype),
        "q": torch.randn((tokens, nq, head_dim), generator=g).to(dtype),
        "k": torch.randn((tokens, nkv, head_dim), generator=g).to(dtype),
        "gate": torch.randn((tokens, inter), generator=g).to(dtype),
        "up": torch.randn((tokens, inter), generator=g).to(dtype),
        "wa": (1 + 0.02 * torch.randn((layers, hidden), generator=g)).to(dtype),
        "wf": (1 + 0.02 * torch.randn((layers, hidden), generator=g)).to(dtype),
        "layers": layers,
        "tokens": tokens,
    }


def run_chain(d: dict, inv_freq, eps: float = 1e-5) -> float:
    """One pass of embedding + layers + final norm; returns wall seconds."""
    inv = torch.as_tensor(inv_freq, dtype=torch.float32)
    t0 = time.perf_counter()
    h = embedding(d["ids"], d["table"])
    q, k = d["q"], d["k"]
    for l in range(d["layers"]):
        h, _, q, k, _ = layer_chain(h, d["attn_out"], d["ffn_out"], q, k, d["gate"], d["up"], d["wa"][l], d["wf"][l],
                                    d["positions"], inv, eps, l == 0)
    add_rmsnorm(h, d["ffn_out"], d["wf"][-1], eps)
    return time.perf_counter() - t0
