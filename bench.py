#!/usr/bin/env python3
"""Benchmark of the B200 per-layer elementwise hot path.

Workload (one "step"): Llama-3.1-8B prefill-shaped elementwise chain in BF16 —
16 sequences x 2048 tokens (32768 tokens, positions 0..2047 per sequence),
hidden 4096, 32/8 heads of 128, intermediate 14336, vocab 128256, 32 layers:
embedding gather, then per layer fused residual-add+RMSNorm, RoPE on Q and K
(llama3 scaling: factor 8, low/high freq 1/4, original context 8192), fused
residual-add+RMSNorm, SwiGLU silu*mul; a final fused add+norm. Activations are
synthetic N(0,1) with 0.1% of the channels scaled x20; the GEMM outputs that
feed the chain (o_proj, down_proj, q/k, gate/up) are synthetic tensors of their
real shapes. Every tensor the chain streams is larger than L2, so no L2 flush
is needed between steps. A timed step is one replay of the step's 130 launches
captured as one CUDA graph; the same steps launched one kernel at a time from
the host are in the line as ``eager``.

Multi-GPU (``torchrun --nproc-per-node N bench.py --gpus N``): the job's 16
sequences are split over the ranks (16/N per GPU; sequences are independent, so
there is no data-path collective); value = the job's 32768 tokens / the slowest
rank's time ("strong" scaling). The line also carries ``weak_scaling``, where
every rank runs its own 16 x 2048 tokens.

At N > 1 (or with ``--pipeline``) the line also carries ``pipeline_config5``:
BASELINE config 5 (70B shapes, 80 layers split into N pipeline stages, NCCL
handoff between stages), with the stage compute and the handoff timed apart.

The same line carries ``tq_config4``: BASELINE config 4 (TurboQuant K+V of
65536 tokens x 8 KV heads x 128 quantized into a paged cache and dequantized
back, 3 and 4 bits), timed per step with CUDA events, the token range split by
16-token blocks across the ranks (strong scaling, max-over-ranks time).

``--impl reference`` times the reference's CPU numerical path (the PyTorch
math of its validation scripts, ``oracle/cpu_chain.py``) on the host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "fused-op tokens/s and achieved HBM GB/s (% of peak) at 1/2/4/8 B200"
T_SEQ, N_SEQ = 2048, 16
HID, NQ, NKV, HD, INTER, LAYERS, VOCAB = 4096, 32, 8, 128, 14336, 32, 128256
ROPE = dict(theta=500000.0, factor=8.0, low=1.0, high=4.0, orig=8192)
EPS = 1e-5
WORKLOAD = "config3: Llama-3.1-8B prefill-shaped elementwise chain (embedding + 32 x [add+rmsnorm, rope q/k, add+rmsnorm, silu*mul] + final add+norm)"


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


# ── clocks sampler ───────────────────────────────────────────────────────────

class Clocks:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.dev)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ── our arm ──────────────────────────────────────────────────────────────────

def run_ours(args, rank: int, world: int, local_rank: int) -> dict | None:
    import numpy as np
    import torch
    import torch.distributed as dist

    from fracture_b200 import kernels as K
    from fracture_b200 import shards
    from fracture_b200.backend import FB_BF16, CudaBackend

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    bf = torch.bfloat16
    stream = torch.cuda.current_stream(dev)
    s = stream.cuda_stream
    freqs = torch.from_numpy(K.rope_freqs_llama3(HD, ROPE["theta"], ROPE["factor"], ROPE["low"], ROPE["high"],
                                                 ROPE["orig"])).to(dev)
    B = 2

    def barrier():
        if world > 1:
            dist.barrier()

    def chain_data(n_seq: int) -> dict:
        T = T_SEQ * n_seq
        g = torch.Generator(device=dev).manual_seed(1234 + rank)

        def act(shape):
            x = torch.randn(shape, generator=g, device=dev)
            cols = torch.rand(shape[-1], generator=g, device=dev) < 0.001  # outlier channels x20
            return torch.where(cols, x * 20.0, x).to(bf)

        d = {"T": T, "n_seq": n_seq,
             "table": (torch.randn((VOCAB, HID), generator=g, device=dev) * 0.02).to(bf),
             "ids": torch.randint(0, VOCAB, (T,), generator=g, device=dev, dtype=torch.int32),
             "positions": (torch.arange(T, device=dev, dtype=torch.int32) % T_SEQ).contiguous(),
             "h": torch.empty((T, HID), device=dev, dtype=bf)}
        d["normed"] = torch.empty_like(d["h"])
        d["attn_proj"], d["ffn_out"] = act((T, HID)), act((T, HID))
        d["q"], d["k"] = act((T, NQ, HD)), act((T, NKV, HD))
        d["gate"], d["up"] = act((T, INTER)), act((T, INTER))
        d["mid"] = torch.empty_like(d["gate"])
        d["wa"] = (1 + 0.02 * torch.randn((LAYERS, HID), generator=g, device=dev)).to(bf)
        d["wf"] = (1 + 0.02 * torch.randn((LAYERS + 1, HID), generator=g, device=dev)).to(bf)
        return d

    def step_bytes(T: int) -> dict:
        # algorithmic bytes (each input read once, each output written once; weight rows once per launch)
        by = {"embed": T * HID * B * 2 + T * 4, "norm": T * HID * B * 2 + HID * B,
              "addnorm": T * HID * B * 4 + HID * B, "rope": T * (NQ + NKV) * HD * B * 2 + T * 4 + HD // 2 * 4,
              "silu": T * INTER * B * 3}
        by["step"] = by["embed"] + by["norm"] + (2 * LAYERS - 1) * by["addnorm"] + LAYERS * by["rope"] \
            + LAYERS * by["silu"] + by["addnorm"]
        return by

    launches_per_step = 1 + 1 + (2 * LAYERS - 1) + LAYERS + LAYERS + 1

    def step(d, st, silu_events=None):
        """One step of the chain on the raw stream handle ``st``; with ``silu_events`` (a list of
        LAYERS event pairs), each silu_mul launch is bracketed by its pair."""
        h, normed = d["h"], d["normed"]
        K.embedding(h, d["table"], d["ids"], stream=st)
        for l in range(LAYERS):
            if l == 0:
                K.rmsnorm(normed, h, d["wa"][0], EPS, stream=st)
            else:
                K.add_rmsnorm(h, d["ffn_out"], d["wa"][l], normed, EPS, stream=st)
            K.rope(d["q"], d["k"], d["positions"], freqs, stream=st)
            K.add_rmsnorm(h, d["attn_proj"], d["wf"][l], normed, EPS, stream=st)
            if silu_events is not None:
                silu_events[l][0].record()
                K.silu_mul(d["mid"], d["gate"], d["up"], stream=st)
                silu_events[l][1].record()
            else:
                K.silu_mul(d["mid"], d["gate"], d["up"], stream=st)
        K.add_rmsnorm(h, d["ffn_out"], d["wf"][LAYERS], normed, EPS, stream=st)

    def capture(d):
        """One step captured as a CUDA graph (its 130 launches replay with no host work between
        them), with external timing events around each silu_mul launch that record on every
        replay."""
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            step(d, side.cuda_stream)  # one eager pass on the capture stream before capture
        stream.wait_stream(side)
        torch.cuda.synchronize(dev)
        ev = [(torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
              for _ in range(LAYERS)]
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            step(d, side.cuda_stream, ev)
        return g, ev

    def timed_chain(d, clocks=None):
        """W untimed steps, then K steps between events, barrier + sync on both sides; the max over
        ranks of the elapsed time and the silu_mul launch times of the last timed step. A step is
        one replay of the captured graph; the same K steps launched one kernel at a time from the
        host (eager) are timed after it for comparison."""
        g, ev = capture(d)

        def run(fn, clk=None):
            for _ in range(args.warmup):
                fn()
            torch.cuda.synchronize(dev)
            barrier()
            torch.cuda.synchronize(dev)
            if clk:
                clk.start()
                time.sleep(0.3)
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            for _ in range(args.steps):
                fn()
            t1.record(stream)
            torch.cuda.synchronize(dev)
            clock = clk.stop() if clk else None
            barrier()
            torch.cuda.synchronize(dev)
            return shards.max_over_ranks(t0.elapsed_time(t1), dev), clock

        ms, clock = run(g.replay, clocks)
        silu = [a.elapsed_time(b) for a, b in ev]
        del g
        ms_eager, _ = run(lambda: step(d, s))
        return ms, silu, clock, ms_eager

    # Headline: the configured job of 16 x 2048 tokens, its sequences split over the ranks
    # (strong scaling: 16/N sequences per GPU, no collective on the data path).
    my_seqs = shards.sequence_shard(N_SEQ, world, rank)
    d = chain_data(len(my_seqs))
    T = d["T"]
    by = step_bytes(T)
    clocks = Clocks(local_rank)
    elapsed_ms, silu_ms, clock, eager_ms = timed_chain(d, clocks)

    # ── e2e through the reference-facing backend API (host buffers) ──
    be = CudaBackend(local_rank)
    be.precompute_rope_freqs_llama3(HD, ROPE["theta"], ROPE["factor"], ROPE["low"], ROPE["high"], ROPE["orig"])
    reg = lambda t_, shape: be.register_external(t_.data_ptr(), shape, FB_BF16)
    Th, Tn = reg(d["h"], (T, HID)), reg(d["normed"], (T, HID))
    Ta, Tf = reg(d["attn_proj"], (T, HID)), reg(d["ffn_out"], (T, HID))
    Tq, Tk = reg(d["q"], (T, NQ, HD)), reg(d["k"], (T, NKV, HD))
    Tg, Tu, Tm = reg(d["gate"], (T, INTER)), reg(d["up"], (T, INTER)), reg(d["mid"], (T, INTER))
    Ttab = reg(d["table"], (VOCAB, HID))
    Twa = [reg(d["wa"][l], (HID,)) for l in range(LAYERS)]
    Twf = [reg(d["wf"][l], (HID,)) for l in range(LAYERS + 1)]
    ns = d["n_seq"]
    last = be.alloc((ns, HID), FB_BF16)
    host_ids = np.random.default_rng(rank).integers(0, VOCAB, T).astype(np.uint32)
    pos_sets = [np.tile(np.arange(T_SEQ, dtype=np.uint32), ns), np.tile(np.arange(1, T_SEQ + 1, dtype=np.uint32), ns)]
    out_host = np.empty(ns * HID * 2, dtype=np.uint8)

    def e2e_step(i):
        pos = pos_sets[i % 2]  # a new forward: positions change, uploaded once, reused by all 32 layers
        be.embedding(host_ids, Ttab, Th)
        for l in range(LAYERS):
            if l > 0:
                be.add(Th, Tf, Th)
            be.rmsnorm(Th, Twa[l], EPS, Tn)
            be.rope(Tq, Tk, pos, ROPE["theta"], HD)
            be.add(Th, Ta, Th)
            be.rmsnorm(Th, Twf[l], EPS, Tn)
            be.silu_mul(Tg, Tu, Tm)
        be.add(Th, Tf, Th)
        be.rmsnorm(Th, Twf[LAYERS], EPS, Tn)
        for sq in range(ns):
            be.copy_rows(Tn, last, sq * T_SEQ + T_SEQ - 1, sq, 1)
        be.copy_to_host(last, out_host)  # synchronous: the step's result is on the host

    e2e_steps = 0 if args.no_e2e else max(3, min(args.steps, 10))
    for i in range(0 if args.no_e2e else max(2, args.warmup)):
        e2e_step(i)
    barrier()
    torch.cuda.synchronize(dev)
    w0 = time.perf_counter()
    for i in range(e2e_steps):
        e2e_step(i)
    e2e_s = shards.max_over_ranks(time.perf_counter() - w0, dev)
    be.close()
    del d

    # The weak-scaling variant (every rank its own 16 x 2048 tokens), kept as a second figure.
    weak = None
    if world > 1:
        dw = chain_data(N_SEQ)
        ms_w, _, _, _ = timed_chain(dw)
        del dw
        ms_step_w = ms_w / args.steps
        weak = {"tokens_per_gpu": T_SEQ * N_SEQ, "ms_per_step": round(ms_step_w, 4),
                "value": round(world * T_SEQ * N_SEQ / (ms_step_w / 1e3), 1), "unit": "tokens/s",
                "frac_of_peak_per_gpu": round(step_bytes(T_SEQ * N_SEQ)["step"] / (ms_step_w / 1e3) / 1e9
                                              / peaks()["hbm_gbs"], 4)}

    if rank != 0:
        return None
    pk = peaks()
    ms_step = elapsed_ms / args.steps
    value = T_SEQ * N_SEQ / (ms_step / 1e3)  # the whole job's tokens over the slowest rank's time
    silu_avg = statistics.mean(silu_ms)
    achieved = by["silu"] / (silu_avg / 1e3) / 1e9
    traffic = None  # DRAM bytes per launch from the committed ncu capture of this kernel at this size
    tf = ROOT / "profiles" / "silu_mul_bf16_config3.md"
    if tf.exists() and world == 1:
        import re

        m = re.search(r"traffic_bytes_per_launch:\s*(\d+)", tf.read_text())
        traffic = int(m.group(1)) if m else None
    res = {
        "metric": METRIC,
        "value": round(value, 1),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) activations, 0.1% channels x20; random-init norm weights and embedding table)",
        "config": {"workload": WORKLOAD, "tokens": T_SEQ * N_SEQ, "sequences": N_SEQ, "tokens_per_gpu": T,
                   "sequences_per_gpu": len(my_seqs), "seq_len": T_SEQ,
                   "hidden": HID, "heads": f"{NQ}/{NKV}x{HD}", "intermediate": INTER, "layers": LAYERS,
                   "vocab": VOCAB, "rope": "llama3 factor 8, low 1, high 4, original 8192, theta 5e5",
                   "parallelism": f"dp{world} (the 16 sequences split over the GPUs, no collective on the data path)",
                   "l2": "each step streams far more than the 126 MB L2 (no flush needed)"},
        "hbm": {"algorithmic_bytes_per_step_per_gpu": by["step"],
                "achieved_gbs_per_gpu": round(by["step"] / (ms_step / 1e3) / 1e9, 1),
                "frac_of_peak": round(by["step"] / (ms_step / 1e3) / 1e9 / pk["hbm_gbs"], 4),
                "peak_gbs": pk["hbm_gbs"], "peak_source": pk["source"]},
        "roofline": {"kernel": "silu_mul_vec_kernel<bf16> (50% of the step's bytes)", "bound": "hbm",
                     "achieved": round(achieved, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / pk["hbm_gbs"], 4), "traffic": traffic,
                     "algorithmic_bytes_per_launch": by["silu"], "avg_launch_ms": round(silu_avg, 5),
                     "peak_source": pk["source"]},
        "e2e": {"value": round(T_SEQ * N_SEQ / (e2e_s / e2e_steps), 1) if e2e_steps else None, "unit": "tokens/s",
                "h2d_bytes_per_step": int(host_ids.nbytes + pos_sets[0].nbytes),
                "d2h_bytes_per_step": int(out_host.nbytes),
                "path": "fracture_b200.backend.CudaBackend (C-ABI Backend mirror): embedding/add/rmsnorm/rope/silu_mul, "
                        "host token ids + positions uploaded each step, last-token rows read back"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clock,
        "timing": "a step is one replay of the step's 130 launches captured as one CUDA graph; the silu_mul times "
                  "come from external events inside the graph (last timed step, 32 launches)",
        "eager": {"ms_per_step": round(eager_ms / args.steps, 4),
                  "value": round(T_SEQ * N_SEQ / (eager_ms / args.steps / 1e3), 1), "unit": "tokens/s",
                  "note": "the same K steps launched one kernel at a time from the host"},
    }
    if weak is not None:
        res["weak_scaling"] = weak
    return res


def run_config2(args, local_rank: int) -> dict:
    """Llama-3.1-8B decode-shaped fused ops in FP16 on one GPU — 64 single tokens
    at positions uniform in [0, 8192): embedding gather, then 32 x [add+RMSNorm, RoPE (llama3),
    add+RMSNorm, silu*mul] and a final add+RMSNorm (130 launches). Every tensor but the embedding
    table fits in L2, so this shape is bound by launch latency, not HBM: it is timed both as eager
    launches and as one captured CUDA graph per step."""
    import torch

    from fracture_b200 import kernels as K

    dev = torch.device("cuda", local_rank)
    T, f16 = 64, torch.float16
    g = torch.Generator(device=dev).manual_seed(2)
    table = (torch.randn((VOCAB, HID), generator=g, device=dev) * 0.02).to(f16)
    ids = torch.randint(0, VOCAB, (T,), generator=g, device=dev, dtype=torch.int32)
    positions = torch.randint(0, 8192, (T,), generator=g, device=dev, dtype=torch.int32)
    h, normed = torch.empty((T, HID), device=dev, dtype=f16), torch.empty((T, HID), device=dev, dtype=f16)
    attn_proj, ffn_out = (torch.randn((T, HID), generator=g, device=dev).to(f16) for _ in range(2))
    q = torch.randn((T, NQ, HD), generator=g, device=dev).to(f16)
    k = torch.randn((T, NKV, HD), generator=g, device=dev).to(f16)
    gate, up = (torch.randn((T, INTER), generator=g, device=dev).to(f16) for _ in range(2))
    mid = torch.empty_like(gate)
    wa = (1 + 0.02 * torch.randn((LAYERS, HID), generator=g, device=dev)).to(f16)
    wf = (1 + 0.02 * torch.randn((LAYERS + 1, HID), generator=g, device=dev)).to(f16)
    freqs = torch.from_numpy(K.rope_freqs_llama3(HD, ROPE["theta"], ROPE["factor"], ROPE["low"], ROPE["high"],
                                                 ROPE["orig"])).to(dev)
    B = 2
    by = (T * HID * B * 2 + T * 4) + (T * HID * B * 2 + HID * B) + (2 * LAYERS - 1 + 1) * (T * HID * B * 4 + HID * B) \
        + LAYERS * (T * (NQ + NKV) * HD * B * 2 + T * 4 + HD // 2 * 4) + LAYERS * T * INTER * B * 3
    launches = 1 + 1 + (2 * LAYERS - 1) + LAYERS + LAYERS + 1

    def chain():
        K.embedding(h, table, ids)
        for l in range(LAYERS):
            if l == 0:
                K.rmsnorm(normed, h, wa[0], EPS)
            else:
                K.add_rmsnorm(h, ffn_out, wa[l], normed, EPS)
            K.rope(q, k, positions, freqs)
            K.add_rmsnorm(h, attn_proj, wf[l], normed, EPS)
            K.silu_mul(mid, gate, up)
        K.add_rmsnorm(h, ffn_out, wf[LAYERS], normed, EPS)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / args.steps

    ms_eager = timed(chain)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        chain()  # one eager pass on the capture stream before capture
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        chain()
    ms_graph = timed(graph.replay)
    del graph
    out = {"workload": "config2: Llama-3.1-8B decode-shaped fused ops, FP16, 64 tokens at positions U[0,8192), "
                       "32 layers of [add+rmsnorm, rope q/k (llama3), add+rmsnorm, silu*mul] + embedding + final norm",
           "tokens": T, "launches_per_step": launches, "algorithmic_bytes_per_step": by,
           "bound": "launch latency (every tensor but the embedding table stays in the 126 MB L2)"}
    for name, ms in (("eager", ms_eager), ("cuda_graph", ms_graph)):
        out[name] = {"ms_per_step": round(ms, 4), "tokens_per_s": round(T / (ms / 1e3), 1),
                     "us_per_launch": round(ms * 1e3 / launches, 3),
                     "effective_gbs": round(by / (ms / 1e3) / 1e9, 1)}
    return out


C5 = dict(hidden=8192, nq=64, nkv=8, hd=128, inter=28672, vocab=128256, layers=80, seqs=256, prompt=1024,
          decode=128, mb_seqs=8, bits=4)


def run_config5(args, rank: int, world: int, local_rank: int) -> dict | None:
    """Llama-3-70B-shaped pipeline, BF16, 80 layers split over the N ranks
    (stage s = rank s). Prefill: 256 sequences x 1024 tokens in micro-batches of 8 sequences,
    hidden states [8192 tokens, 8192] handed stage to stage by NCCL send/recv (fracture_b200.shards).
    Decode: 128 steps for the 256 sequences in N groups, as a ring (the last stage hands each group's
    next tokens back to stage 0). Per layer: fused add+RMSNorm, RoPE q/k (64/8 heads), fused
    add+RMSNorm, silu*mul (I = 28672) and a 4-bit TurboQuant write of K and V into this stage's
    paged cache (slot-mapped, one launch each). The GEMMs between these ops are outside the path:
    synthetic tensors of their shapes stand in for their outputs."""
    import torch

    from fracture_b200 import kernels as K
    from fracture_b200 import shards

    c = C5
    dev = torch.device("cuda", local_rank)
    bf = torch.bfloat16
    H, NQ5, NKV5, HD5, I5 = c["hidden"], c["nq"], c["nkv"], c["hd"], c["inter"]
    my_layers = shards.stage_layers(c["layers"], world, rank)
    nl = len(my_layers)
    g = torch.Generator(device=dev).manual_seed(500 + rank)
    mb_tokens = c["mb_seqs"] * c["prompt"]
    n_mb = c["seqs"] // c["mb_seqs"]
    seq_rows = c["prompt"] + c["decode"]  # pool rows per sequence (blocks of 16, contiguous per sequence)
    bits = c["bits"]
    P = HD5 * bits // 8

    def act(shape):
        return torch.randn(shape, generator=g, device=dev).to(bf)

    # stand-ins for the GEMM outputs, shared by all layers of this stage
    attn_out, ffn_out = act((mb_tokens, H)), act((mb_tokens, H))
    q, k, v = act((mb_tokens, NQ5, HD5)), act((mb_tokens, NKV5, HD5)), act((mb_tokens, NKV5, HD5))
    gate, up = act((mb_tokens, I5)), act((mb_tokens, I5))
    mid = torch.empty_like(gate)
    normed = torch.empty((mb_tokens, H), device=dev, dtype=bf)
    wa = (1 + 0.02 * torch.randn((nl, H), generator=g, device=dev)).to(bf)
    wf = (1 + 0.02 * torch.randn((nl + 1, H), generator=g, device=dev)).to(bf)
    table = (torch.randn((c["vocab"], H), generator=g, device=dev) * 0.02).to(bf) if rank == 0 else None
    freqs = torch.from_numpy(K.rope_freqs_llama3(HD5, ROPE["theta"], ROPE["factor"], ROPE["low"], ROPE["high"],
                                                 ROPE["orig"])).to(dev)
    rots = [torch.from_numpy(K.tq_rotation_matrix(HD5, sd)).to(dev) for sd in (42, 542)]
    cen = torch.from_numpy(K.tq_codebook(HD5, bits)[0]).to(dev)
    rows = c["seqs"] * seq_rows
    pools = [[(torch.empty((rows, NKV5 * P), dtype=torch.uint8, device=dev),
               torch.empty((rows, NKV5), dtype=torch.float16, device=dev)) for _ in range(2)] for _ in range(nl)]
    pos_prefill = (torch.arange(mb_tokens, device=dev, dtype=torch.int32) % c["prompt"]).contiguous()
    ids_prefill = torch.randint(0, c["vocab"], (n_mb, mb_tokens), generator=g, device=dev, dtype=torch.int32)
    # slot of token t of prefill micro-batch m: sequence (m * mb_seqs + t // prompt), position t % prompt
    tt = torch.arange(mb_tokens, device=dev, dtype=torch.int64)
    slots_prefill = [((m * c["mb_seqs"] + tt // c["prompt"]) * seq_rows + tt % c["prompt"]).contiguous()
                     for m in range(n_mb)]
    hbuf = [torch.empty((mb_tokens, H), device=dev, dtype=bf) for _ in range(2)]
    # the layers work in place on the received buffer, which is then sent on: three receive
    # buffers keep the receive of m + 1 off the buffer whose send (m - 1) may still be in flight
    rbuf = [torch.empty((mb_tokens, H), device=dev, dtype=bf) for _ in range(3)]

    def layers(h, T, pos, slots, li0=0):
        for j in range(nl):
            K.add_rmsnorm(h, attn_out[:T], wa[j], normed[:T], EPS)
            K.rope(q[:T], k[:T], pos, freqs)
            K.tq_compress_kv_slots(k[:T], v[:T], rots[0], rots[1], cen, cen, bits, bits, pools[j][0][0],
                                   pools[j][0][1], pools[j][1][0], pools[j][1][1], slots)
            K.add_rmsnorm(h, ffn_out[:T], wf[j], normed[:T], EPS)
            K.silu_mul(mid[:T], gate[:T], up[:T])

    link = shards.StageLink(rank, world)

    def prefill():
        def first_input(m):
            K.embedding(hbuf[m % 2], table, ids_prefill[m])
            return hbuf[m % 2]

        def stage(m, x):
            layers(x, mb_tokens, pos_prefill, slots_prefill[m])
            if rank == world - 1:
                K.add_rmsnorm(x, ffn_out, wf[nl], normed, EPS)
            return x

        shards.run_pipeline(n_mb, link, first_input, stage, rbuf)

    # decode: G groups of sequences in flight around the ring; each group's layer stack on this
    # stage is one captured CUDA graph (positions and slots live in static tensors updated per step)
    G = max(world, 1)
    gs = c["seqs"] // G
    ring = shards.StageLink(rank, world, ring=True)
    ids_dec = [torch.randint(0, c["vocab"], (gs,), generator=g, device=dev, dtype=torch.int32) for _ in range(G)]
    hdec = [torch.empty((gs, H), device=dev, dtype=bf) for _ in range(G)]
    pos_dec = torch.empty((gs,), device=dev, dtype=torch.int32)
    slot_base = torch.arange(c["seqs"], device=dev, dtype=torch.int64).view(G, gs) * seq_rows
    slots_dec = torch.empty((G, gs), device=dev, dtype=torch.int64)
    graphs = []
    replay_events = []

    def group_body(gr):
        layers(hdec[gr], gs, pos_dec, slots_dec[gr])
        if rank == world - 1:
            K.add_rmsnorm(hdec[gr], ffn_out[:gs], wf[nl], normed[:gs], EPS)

    def decode():
        import torch.distributed as dist

        h_send = [None] * G    # send of hdec[gr] to the next stage still in flight
        ids_send = [None] * G  # ring send of ids_dec[gr] still in flight
        for t in range(c["decode"]):
            pos_dec.fill_(c["prompt"] + t)
            torch.add(slot_base, c["prompt"] + t, out=slots_dec)
            for gr in range(G):
                h = hdec[gr]
                if h_send[gr] is not None:  # hdec[gr] is about to be overwritten
                    h_send[gr].wait()
                    h_send[gr] = None
                if rank == 0:
                    if t > 0 and world > 1:
                        ring.irecv(ids_dec[gr]).wait()
                    K.embedding(h, table, ids_dec[gr])
                else:
                    link.irecv(h).wait()
                if graphs:
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    graphs[gr].replay()
                    e1.record()
                    replay_events.append((e0, e1))
                else:
                    group_body(gr)
                if rank < world - 1:
                    h_send[gr] = link.isend(h)
                else:
                    if ids_send[gr] is not None:
                        ids_send[gr].wait()
                        ids_send[gr] = None
                    # next tokens of the group (a deterministic stand-in for sampling)
                    ids_dec[gr].add_(1).remainder_(c["vocab"])
                    if world > 1 and t + 1 < c["decode"]:
                        ids_send[gr] = ring.isend(ids_dec[gr])
        for w_ in h_send + ids_send:
            if w_ is not None:
                w_.wait()
        if world > 1:
            dist.barrier()

    def capture_decode_graphs():
        torch.cuda.synchronize(dev)
        for gr in range(G):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                group_body(gr)
            graphs.append(graph)
        torch.cuda.synchronize(dev)

    def timed(fn, reps):
        fn()  # warm-up pass
        torch.cuda.synchronize(dev)
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        return shards.max_over_ranks(e0.elapsed_time(e1) / reps, dev)

    reps = max(1, min(args.steps, 2))
    ms_pre = timed(prefill, reps)

    # Where the prefill time goes. (1) Stage compute alone: one micro-batch through this stage's
    # layers, no handoff. (2) The handoff alone: every boundary moves one micro-batch at once
    # (stage s -> s + 1), nothing else running. The pipelined prefill is compared with
    # (micro-batches + stages - 1) x the slowest stage's compute, its bubble included.
    def compute_only():
        layers(rbuf[0], mb_tokens, pos_prefill, slots_prefill[0])

    ms_compute = timed(compute_only, 4)
    handoff = None
    if world > 1:
        import torch.distributed as dist

        def boundary_exchange():
            ops = []
            if rank < world - 1:
                ops.append(dist.P2POp(dist.isend, rbuf[1], rank + 1))
            if rank > 0:
                ops.append(dist.P2POp(dist.irecv, rbuf[2], rank - 1))
            for w_ in dist.batch_isend_irecv(ops):
                w_.wait()

        ms_handoff = timed(boundary_exchange, 8)
        mb_bytes = mb_tokens * H * 2
        handoff = {"bytes_per_microbatch": mb_bytes, "ms_per_microbatch": round(ms_handoff, 4),
                   "gbs_per_boundary": round(mb_bytes / (ms_handoff / 1e3) / 1e9, 1),
                   "peer_copy_reference_gbs": 770.0,
                   "all_microbatches_ms": round(ms_handoff * n_mb, 3),
                   "bytes_per_boundary": n_mb * mb_bytes}
    ideal_pre = (n_mb + world - 1) * ms_compute

    decode()  # eager pass: sizes every workspace before capture
    capture_decode_graphs()
    replay_events.clear()
    ms_dec = timed(decode, 1)
    graphs.clear()
    # the timed pass is the second decode() call inside timed(): the last n_replays events
    n_replays = c["decode"] * G
    replay_ms = sum(e0.elapsed_time(e1) for e0, e1 in replay_events[-n_replays:])
    replay_events.clear()
    replay_ms = shards.max_over_ranks(replay_ms, dev)
    # algorithmic bytes per token per layer (BF16 activations; 4-bit K and V into the pool)
    by_tok_layer = 2 * (4 * H * 2) + (NQ5 + NKV5) * HD5 * 2 * 2 + 4 + 3 * I5 * 2 \
        + 2 * (NKV5 * HD5 * 2 + NKV5 * (P + 2) + 8)
    pre_tokens = c["seqs"] * c["prompt"]
    dec_tokens = c["seqs"] * c["decode"]
    stage_bytes_pre = by_tok_layer * nl * pre_tokens
    if rank != 0:
        return None
    pk = peaks()
    return {"workload": "config5: Llama-3-70B-shaped pipeline, BF16, 80 layers split over the GPUs; per layer "
                        "add+rmsnorm, rope q/k (64/8 heads), add+rmsnorm, silu*mul (I=28672) and 4-bit TurboQuant "
                        "K+V writes into a paged cache; 256 x 1024 prefill in micro-batches of 8 sequences, "
                        "then 128 decode steps in groups around a ring",
            "stages": world, "layers_per_stage": nl, "micro_batch_tokens": mb_tokens,
            "handoff": "NCCL send/recv of BF16 hidden states between neighbouring stages (decode: next tokens "
                       "from the last stage back to stage 0)" if world > 1 else "none (one stage)",
            "prefill": {"ms": round(ms_pre, 3), "tokens_per_s": round(pre_tokens / (ms_pre / 1e3), 1),
                        "micro_batches": n_mb,
                        "stage_algorithmic_bytes": stage_bytes_pre,
                        "stage_achieved_gbs": round(stage_bytes_pre / (ms_pre / 1e3) / 1e9, 1),
                        "stage_frac_of_peak": round(stage_bytes_pre / (ms_pre / 1e3) / 1e9 / pk["hbm_gbs"], 4),
                        "handoff_bytes_per_boundary": pre_tokens * H * 2,
                        "breakdown": {
                            "stage_compute_ms_per_microbatch": round(ms_compute, 4),
                            "stage_compute_gbs": round(by_tok_layer * nl * mb_tokens / (ms_compute / 1e3) / 1e9, 1),
                            "pipelined_ideal_ms": round(ideal_pre, 3),
                            "pipeline_overhead_ms": round(ms_pre - ideal_pre, 3),
                            "handoff_alone": handoff,
                            "note": "ideal = (micro-batches + stages - 1) x the slowest stage's compute per "
                                    "micro-batch (bubble included); overhead = measured - ideal is the exposed "
                                    "cost of the handoffs and of stage imbalance"}},
            "decode": {"ms": round(ms_dec, 3), "tokens_per_s": round(dec_tokens / (ms_dec / 1e3), 1),
                       "groups": G, "group_sequences": gs,
                       "breakdown": {"graph_replay_ms_busiest_stage": round(replay_ms, 3),
                                     "outside_graphs_ms": round(ms_dec - replay_ms, 3),
                                     "note": "graph replays = the stage's layers (device time between events "
                                             "around each replay, summed); the rest of the decode time is the "
                                             "handoff waits, embedding and launch gaps"},
                       "launch": "one CUDA graph per group and stage per step (layers of the stage); NCCL "
                                 "handoffs and the embedding outside the graphs"},
            "peak_gbs": pk["hbm_gbs"], "peak_source": pk["source"]}


def run_tq_config4(args, rank: int, world: int, local_rank: int) -> dict | None:
    """TurboQuant K and V of [65536 tokens, 8 KV heads, 128] FP16 (N(0,1), 0.5% of
    elements x10) quantized into a paged cache (block 16, random block table) and dequantized back,
    at 3 and 4 bits. The 65536 tokens are split by 16-token blocks across the ranks (each rank owns
    a disjoint pool shard; strong scaling, no collective on the data path). One step = K and V."""
    import torch
    import torch.distributed as dist

    from fracture_b200 import kernels as K

    dev = torch.device("cuda", local_rank)
    from fracture_b200 import shards

    T_all, H, D = 65536, NKV, HD
    T = len(shards.block_shard(T_all, world, rank))
    g = torch.Generator(device=dev).manual_seed(99 + rank)
    kv = []
    for _ in range(2):
        x = torch.randn((T, H, D), generator=g, device=dev)
        kv.append(torch.where(torch.rand((T, H, D), generator=g, device=dev) < 0.005, x * 10.0, x).to(torch.float16))
    rot = [torch.from_numpy(K.tq_rotation_matrix(D, sd)).to(dev) for sd in (42, 542)]
    table = torch.randperm(T // 16, generator=g, device=dev).to(torch.int32)
    outs = [torch.empty((T, H, D), dtype=torch.float16, device=dev) for _ in range(2)]
    stream = torch.cuda.current_stream(dev)
    pk = peaks()
    res = {}

    # A shard can fit in the 126 MB L2 (2 x 67 MB at 2 GPUs, less beyond): every timed step starts
    # after a 256 MB write that evicts it, and only the step itself is inside the events.
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for e0, e1 in ev:
            flush.fill_(1)
            e0.record(stream)
            fn()
            e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = sum(e0.elapsed_time(e1) for e0, e1 in ev) / args.steps
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    for bits in (4, 3):
        P = D * bits // 8
        cen = torch.from_numpy(K.tq_codebook(D, bits)[0]).to(dev)
        pools = [(torch.empty((T, H * P), dtype=torch.uint8, device=dev),
                  torch.empty((T, H), dtype=torch.float16, device=dev)) for _ in range(2)]

        def quant():  # K and V of the step in one call (one launch)
            K.tq_compress_kv_paged(kv[0], kv[1], rot[0], rot[1], cen, cen, bits, bits, pools[0][0], pools[0][1],
                                   pools[1][0], pools[1][1], block_table=table)

        def dequant():  # K and V of the step in one call (one launch)
            K.tq_dequant_kv_paged(pools[0][0], pools[0][1], pools[1][0], pools[1][1], rot[0], rot[1], cen, cen, bits,
                                  bits, outs[0], outs[1], block_table=table)

        ms_q, ms_d = timed(quant), timed(dequant)
        vec = 2 * T_all * H  # K and V vectors of the whole job
        by_q = vec * (D * 2 + P + 2) + 2 * (T_all // 16) * 4  # read fp16, write codes + fp16 norm (+ block tables)
        by_d = vec * (P + 2 + D * 2) + 2 * (T_all // 16) * 4
        for name, ms, by in (("quantize", ms_q, by_q), ("dequantize", ms_d, by_d)):
            gbs = by / (ms / 1e3) / 1e9
            res.setdefault(name, {})[f"{bits}bit"] = {
                "ms_per_step": round(ms, 4), "vectors_per_s": round(vec / (ms / 1e3), 1),
                "algorithmic_bytes_per_step": by, "achieved_gbs": round(gbs, 1),
                "frac_of_peak": round(gbs / (world * pk["hbm_gbs"]), 4)}  # of all GPUs' peak
    if rank != 0:
        return None
    return {"workload": "config4: TurboQuant K+V [65536, 8, 128] FP16 -> paged cache (block 16, random table) "
                        "and back, Lloyd-Max 3/4-bit, per-vector FP16 norms",
            "tokens": T_all, "tokens_per_gpu": T, "scaling": "strong" if world > 1 else None,
            "parallelism": f"token shards of 16-token blocks over {world} GPU(s), no collective on the data path",
            "output_dtype": "fp16", "peak_gbs": pk["hbm_gbs"], "peak_source": pk["source"],
            "frac_of": f"{world} x peak_gbs (whole job)",
            "l2": "256 MB written before every timed step (a shard can fit in L2); the flush is outside the timed events",
            "bound": "hbm", **res}


def run_tq_attention(args, local_rank: int) -> dict:
    """Decode attention over the TurboQuant cache (the consumer of config 4's format): 64
    sequences, one query token each at the end of an 8192-token context, Llama-3.1-8B heads
    (32 Q / 8 KV x 128), keys 4-bit and values 2-bit (the reference's default TurboQuantConfig,
    turboquant.rs:20-30), random block tables over one shared pool. One step = one
    fb_launch_tq_attention_paged call for all 64 sequences. The cache (420 MB) is larger than
    L2, so no flush is needed."""
    import torch

    from fracture_b200 import kernels as K

    dev = torch.device("cuda", local_rank)
    S, L, HQ, HKV, D, KB, VB = 64, 8192, NQ, NKV, HD, 4, 2
    nblk = L // 16
    g = torch.Generator(device=dev).manual_seed(7)
    rows = S * L
    kp = torch.empty((rows, HKV * D * KB // 8), dtype=torch.uint8, device=dev)
    vp = torch.empty((rows, HKV * D * VB // 8), dtype=torch.uint8, device=dev)
    kn = torch.empty((rows, HKV), dtype=torch.float16, device=dev)
    vn = torch.empty((rows, HKV), dtype=torch.float16, device=dev)
    tables = torch.randperm(S * nblk, generator=g, device=dev).to(torch.int32).view(S, nblk)
    pik, piv = (torch.from_numpy(K.tq_rotation_matrix(D, sd)).to(dev) for sd in (42, 542))
    ck, cv = (torch.from_numpy(K.tq_codebook(D, b)[0]).to(dev) for b in (KB, VB))
    for s in range(S):  # fill the cache through the compress kernels
        x = torch.randn((L, HKV, D), generator=g, device=dev).half()
        K.tq_compress_paged(x, pik, ck, KB, kp, kn, block_table=tables[s])
        K.tq_compress_paged(x, piv, cv, VB, vp, vn, block_table=tables[s])
    q = torch.randn((S, 1, HQ, D), generator=g, device=dev).half()
    out = torch.empty_like(q)
    kv_lens = torch.full((S,), L, dtype=torch.int32, device=dev)
    starts = torch.full((S,), L - 1, dtype=torch.int32, device=dev)
    ws = torch.empty(K.tq_attention_workspace_bytes(S, 1, HQ, L), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        K.tq_attention_paged(q, kp, kn, vp, vn, tables, kv_lens, starts, pik, piv, ck, cv, KB, VB, out,
                             max_kv_len=L, workspace=ws)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for e0, e1 in ev:
        e0.record(stream)
        step()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = sum(e0.elapsed_time(e1) for e0, e1 in ev) / args.steps
    kv_bytes = S * L * HKV * (D * KB // 8 + 2 + D * VB // 8 + 2)
    by = kv_bytes + 2 * S * HQ * D * 2 + S * nblk * 4 + 2 * D * D * 4
    gbs = by / (ms / 1e3) / 1e9
    pk = peaks()
    return {"workload": "TurboQuant paged attention (decode): 64 sequences x 1 query token, context 8192, "
                        "32 Q / 8 KV heads x 128, K 4-bit / V 2-bit, FP16 queries and output",
            "kernels": "tqa_rotate_q + tqa_stream (persistent CTAs; 4 producer warps feed a ring of stages by TMA, two 16-position blocks x 8 KV heads per stage; 8 consumer warps decode codes through 64 KB-aligned lane-private tables into mma.sync m16n8k16 FP16 operands, FP32 accumulators; split-K over 512-position items at this shape) + tqa_combine",
            "ms_per_step": round(ms, 4), "query_tokens_per_s": round(S / (ms / 1e3), 1),
            "kv_positions_per_s": round(S * L / (ms / 1e3), 1), "algorithmic_bytes_per_step": by,
            "achieved_gbs": round(gbs, 1), "frac_of_peak": round(gbs / pk["hbm_gbs"], 4),
            "peak_gbs": pk["hbm_gbs"], "peak_source": pk["source"],
            "l2": "the 420 MB cache is larger than L2 (no flush)"}


def run_tq_attention_abi(args, local_rank: int, steps: int = 0) -> dict:
    """The reference ABI's call (launch_attention_paged_tq, ffi.rs:251-274: one sequence, FP16,
    per-block pointer arrays), as CudaBackend::attention_paged_tq makes it once per sequence and
    layer: one decode token at the end of a 32768-token context, 32 Q / 8 KV heads x 128, K 4-bit /
    V 2-bit. Twenty layers' caches (26 MB each, 529 MB in all: more than L2) sit in one pool, their
    blocks shuffled and addressed through per-layer pointer arrays; one step = one call, and
    consecutive calls go to consecutive layers, as a decode step's do. Timed as twenty calls (one
    per layer) captured in a CUDA graph and replayed, so that no host time sits between calls (the
    figure is GPU time per call). Codes and norms are random bytes and values: the kernels' work
    does not depend on them."""
    import torch

    from fracture_b200 import _lib
    from fracture_b200 import kernels as K

    dev = torch.device("cuda", local_rank)
    L, HQ, HKV, D, KB, VB, NL = 32768, NQ, NKV, HD, 4, 2, 20
    nblk = L // 16
    Pk, Pv = D * KB // 8, D * VB // 8
    g = torch.Generator(device=dev).manual_seed(11)
    rows = NL * L
    kp = torch.randint(0, 256, (rows, HKV * Pk), dtype=torch.uint8, device=dev, generator=g)
    vp = torch.randint(0, 256, (rows, HKV * Pv), dtype=torch.uint8, device=dev, generator=g)
    kn = (torch.rand((rows, HKV), generator=g, device=dev) + 0.5).half()
    vn = (torch.rand((rows, HKV), generator=g, device=dev) + 0.5).half()
    perm = torch.randperm(NL * nblk, generator=g, device=dev).to(torch.int64)
    pik, piv = (torch.from_numpy(K.tq_rotation_matrix(D, sd)).to(dev) for sd in (42, 542))
    ck, cv = (torch.from_numpy(K.tq_codebook(D, b)[0]).to(dev) for b in (KB, VB))
    layers = []
    for layer in range(NL):  # layer l: its own blocks, block b at entry b of its pointer arrays
        blocks = perm[layer * nblk:(layer + 1) * nblk]
        arr = lambda t, row: t.data_ptr() + blocks * (16 * row)
        layers.append((arr(kp, HKV * Pk), arr(kn, HKV * 2), arr(vp, HKV * Pv), arr(vn, HKV * 2)))
    table = torch.arange(nblk, dtype=torch.int32, device=dev)
    q = torch.randn((1, HQ, D), generator=g, device=dev).half()
    out = torch.empty_like(q)
    lib = _lib.load()
    side = torch.cuda.Stream(dev)

    def call(layer):
        kpa, kna, vpa, vna = layers[layer]
        rc = lib.launch_attention_paged_tq(out.data_ptr(), q.data_ptr(), table.data_ptr(), kpa.data_ptr(),
                                           kna.data_ptr(), vpa.data_ptr(), vna.data_ptr(), pik.data_ptr(),
                                           piv.data_ptr(), ck.data_ptr(), cv.data_ptr(), 1, HQ, HKV, D, L, L - 1,
                                           KB, VB, Pk, Pv, torch.cuda.current_stream(dev).cuda_stream)
        if rc:
            raise RuntimeError(f"launch_attention_paged_tq: {rc}")

    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for i in range(max(args.warmup, 3)):  # the first call sizes the library workspace
            call(i % NL)
    torch.cuda.synchronize(dev)
    if steps:  # profile mode: eager calls only
        for i in range(steps):
            call(i % NL)
        torch.cuda.synchronize(dev)
        return {}
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        for layer in range(NL):
            call(layer)
    graph.replay()
    torch.cuda.synchronize(dev)
    cur = torch.cuda.current_stream(dev)  # replays run on the current stream
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    e0.record(cur)
    for _ in range(reps):
        graph.replay()
    e1.record(cur)
    torch.cuda.synchronize(dev)
    us = e0.elapsed_time(e1) * 1000.0 / (reps * NL)
    by = L * HKV * (Pk + Pv + 4) + 2 * HQ * D * 2 + nblk * (4 + 4 * 8) + 2 * D * D * 4
    del graph
    pk = peaks()
    return {"workload": "reference ABI call (launch_attention_paged_tq): 1 sequence x 1 decode token, context 32768, "
                        "32 Q / 8 KV heads x 128, K 4-bit / V 2-bit, per-block pointer arrays; 20 layers' caches, "
                        "one call per layer in turn",
            "us_per_call": round(us, 2), "algorithmic_bytes_per_call": by,
            "achieved_gbs": round(by / us / 1e3, 1), "frac_of_peak": round(by / us / 1e3 / pk["hbm_gbs"], 4),
            "timing": "20 calls (one per layer, 529 MB of caches: more than L2) in one CUDA graph, 10 replays; "
                      "GPU time per call"}


def run_attention_fp16(args, local_rank: int) -> dict:
    """The same decode attention over the uncompressed FP16 paged cache (PagedKvCacheManager's
    path): 64 sequences x 1 query token at the end of an 8192-token context, 32 Q / 8 KV heads x
    128, one fb_launch_attention_paged call per step. The 2.1 GB cache is larger than L2."""
    import torch

    from fracture_b200 import kernels as K

    dev = torch.device("cuda", local_rank)
    S, L, HQ, HKV, D = 64, 8192, NQ, NKV, HD
    nblk = L // 16
    g = torch.Generator(device=dev).manual_seed(8)
    kp = torch.empty((S * L, HKV, D), dtype=torch.float16, device=dev)
    vp = torch.empty_like(kp)
    tables = torch.randperm(S * nblk, generator=g, device=dev).to(torch.int32).view(S, nblk)
    for s in range(S):
        x = torch.randn((L, HKV, D), generator=g, device=dev).half()
        K.kv_append_paged(x, x, kp, vp, tables[s])
    q = torch.randn((S, 1, HQ, D), generator=g, device=dev).half()
    out = torch.empty_like(q)
    kv_lens = torch.full((S,), L, dtype=torch.int32, device=dev)
    starts = torch.full((S,), L - 1, dtype=torch.int32, device=dev)
    ws = torch.empty(K.attention_workspace_bytes(S, 1, HQ, L), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        K.attention_paged(q, kp, vp, tables, kv_lens, starts, out, max_kv_len=L, workspace=ws)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for e0, e1 in ev:
        e0.record(stream)
        step()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = sum(e0.elapsed_time(e1) for e0, e1 in ev) / args.steps
    by = S * L * HKV * D * 2 * 2 + 2 * S * HQ * D * 2 + S * nblk * 4
    gbs = by / (ms / 1e3) / 1e9
    pk = peaks()
    return {"workload": "paged attention (decode) over the FP16 cache: 64 sequences x 1 query token, context 8192, "
                        "32 Q / 8 KV heads x 128",
            "kernels": "kvp_mma (persistent CTAs, split-K over 2048-position items at this shape, mma.sync m16n8k16 on the cache rows loaded straight into fragment registers, FP32 accumulators) + kvp_combine",
            "ms_per_step": round(ms, 4), "query_tokens_per_s": round(S / (ms / 1e3), 1),
            "kv_positions_per_s": round(S * L / (ms / 1e3), 1), "algorithmic_bytes_per_step": by,
            "achieved_gbs": round(gbs, 1), "frac_of_peak": round(gbs / pk["hbm_gbs"], 4),
            "peak_gbs": pk["hbm_gbs"], "peak_source": pk["source"],
            "l2": "the 2.1 GB cache is larger than L2 (no flush)"}


CPU_TOKENS, CPU_LAYERS = 1024, 8  # the CPU sample both arms time: a slice of the config-3 job


def cpu_sample(warmup: int, reps: int) -> dict:
    """The reference's CPU path (oracle/cpu_chain.py, torch on every host thread) on a bounded sample
    of the config-3 workload: CPU_TOKENS tokens through CPU_LAYERS layers of the chain, with the
    full 128,256-row embedding table. Both the GPU arm's ``cpu_baseline`` and ``--impl reference``
    run this same function, so their numbers differ only by run-to-run noise."""
    import torch

    from oracle import cpu_chain, ops

    n = cpu_chain.set_threads()
    inv = ops.rope_freqs_llama3(HD, ROPE["theta"], ROPE["factor"], ROPE["low"], ROPE["high"], ROPE["orig"])
    data = cpu_chain.make_data(CPU_TOKENS, HID, NQ, NKV, HD, INTER, CPU_LAYERS, VOCAB, torch.bfloat16)
    for _ in range(max(1, warmup)):
        cpu_chain.run_chain(data, inv)
    secs = [cpu_chain.run_chain(data, inv) for _ in range(reps)]
    per_step = statistics.mean(secs) * LAYERS / CPU_LAYERS  # scaled to the 32-layer chain
    value = CPU_TOKENS / per_step
    return {"value": round(value, 2), "unit": "tokens/s", "cores": n, "kind": "port",
            "seconds_per_step": per_step,
            "sample": f"{CPU_TOKENS} tokens x {CPU_LAYERS} layers of the config-3 chain (BF16 storage, f32 math, "
                      f"torch CPU on {n} threads, full {VOCAB}-row embedding table), mean of {reps} runs after "
                      f"{max(1, warmup)} warm-up; tokens/s scaled to the 32-layer chain"}


def cpu_baseline(reps: int = 3) -> dict:
    r = cpu_sample(1, reps)
    r.pop("seconds_per_step")
    return r


def run_reference(args, rank: int) -> dict | None:
    """The reference's CPU path on the host cores; rank 0 only (other ranks exit without work)."""
    if rank != 0:
        return None
    cb = cpu_sample(args.warmup, args.steps)
    per_step = cb.pop("seconds_per_step")
    value = cb["value"]
    return {
        "impl": "reference",
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": 0, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(per_step * 1e3, 2), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "tokens": T_SEQ * N_SEQ, "sequences": N_SEQ, "seq_len": T_SEQ,
                   "hidden": HID, "heads": f"{NQ}/{NKV}x{HD}", "intermediate": INTER, "layers": LAYERS,
                   "vocab": VOCAB, "rope": "llama3 factor 8, low 1, high 4, original 8192, theta 5e5",
                   "tokens_per_step_sample": CPU_TOKENS, "layers_timed": CPU_LAYERS},
        "cpu_baseline": cb,
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def profile_kernel(args) -> None:
    """One kernel at its config-3 size: ``--warmup`` launches then one more (for ``ncu -s W -c 1``)."""
    import torch

    from fracture_b200 import kernels as K

    if args.profile_kernel == "tq_attention_abi":  # W warm-up calls + 1, eager
        run_tq_attention_abi(args, 0, steps=1)
        print(json.dumps({"kernel": args.profile_kernel}))
        return
    if args.profile_kernel in ("tq_attention", "attention_fp16"):  # the bench's workload, W warm-ups + 1
        args.steps = 1
        fn = run_tq_attention if args.profile_kernel == "tq_attention" else run_attention_fp16
        print(json.dumps({"kernel": args.profile_kernel, "ms": fn(args, 0)["ms_per_step"]}))
        return

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7)
    T, bf = T_SEQ * N_SEQ, torch.bfloat16
    rnd = lambda *shape: torch.randn(shape, generator=g, device=dev).to(bf)
    if args.profile_kernel == "silu_mul":
        a, b, o = rnd(T, INTER), rnd(T, INTER), torch.empty((T, INTER), device=dev, dtype=bf)
        fn = lambda: K.silu_mul(o, a, b)
    elif args.profile_kernel == "add_rmsnorm":
        h, r, w, o = rnd(T, HID), rnd(T, HID), rnd(HID), torch.empty((T, HID), device=dev, dtype=bf)
        fn = lambda: K.add_rmsnorm(h, r, w, o, EPS)
    elif args.profile_kernel == "rope":
        q, k = rnd(T, NQ, HD), rnd(T, NKV, HD)
        pos = (torch.arange(T, device=dev, dtype=torch.int32) % T_SEQ)
        f = torch.from_numpy(K.rope_freqs_llama3(HD, ROPE["theta"], ROPE["factor"], ROPE["low"], ROPE["high"],
                                                 ROPE["orig"])).to(dev)
        fn = lambda: K.rope(q, k, pos, f)
    elif args.profile_kernel == "tq_compress":
        # K and V of 65536 tokens x 8 KV heads x 128, FP16, 4-bit, random block
        # table, one launch for both (as the bench's quantize step)
        Tk = 65536
        xs = []
        for _ in range(2):
            x = torch.randn((Tk, NKV, HD), generator=g, device=dev)
            xs.append(torch.where(torch.rand((Tk, NKV, HD), generator=g, device=dev) < 0.005, x * 10, x)
                      .to(torch.float16))
        rots = [torch.from_numpy(K.tq_rotation_matrix(HD, sd)).to(dev) for sd in (42, 542)]
        cen = torch.from_numpy(K.tq_codebook(HD, 4)[0]).to(dev)
        table = torch.randperm(Tk // 16, generator=g, device=dev).to(torch.int32)
        pools = [(torch.empty((Tk, NKV * 64), dtype=torch.uint8, device=dev),
                  torch.empty((Tk, NKV), dtype=torch.float16, device=dev)) for _ in range(2)]
        fn = lambda: K.tq_compress_kv_paged(xs[0], xs[1], rots[0], rots[1], cen, cen, 4, 4, pools[0][0], pools[0][1],
                                            pools[1][0], pools[1][1], block_table=table)
    elif args.profile_kernel == "tq_dequant":
        # BASELINE config 4 dequantize: the K and V pools of 65536 tokens x 8 KV heads x 128 back
        # to FP16, one launch for both (as the bench's dequantize step)
        Tk = 65536
        rots = [torch.from_numpy(K.tq_rotation_matrix(HD, sd)).to(dev) for sd in (42, 542)]
        cen = torch.from_numpy(K.tq_codebook(HD, 4)[0]).to(dev)
        table = torch.randperm(Tk // 16, generator=g, device=dev).to(torch.int32)
        pools = []
        for j in range(2):
            x = torch.randn((Tk, NKV, HD), generator=g, device=dev)
            x = torch.where(torch.rand((Tk, NKV, HD), generator=g, device=dev) < 0.005, x * 10, x).to(torch.float16)
            packed = torch.empty((Tk, NKV * 64), dtype=torch.uint8, device=dev)
            norms = torch.empty((Tk, NKV), dtype=torch.float16, device=dev)
            K.tq_compress_paged(x, rots[j], cen, 4, packed, norms, block_table=table)
            pools.append((packed, norms))
        outs = [torch.empty((Tk, NKV, HD), dtype=torch.float16, device=dev) for _ in range(2)]
        fn = lambda: K.tq_dequant_kv_paged(pools[0][0], pools[0][1], pools[1][0], pools[1][1], rots[0], rots[1], cen,
                                           cen, 4, 4, outs[0], outs[1], block_table=table)
    elif args.profile_kernel in ("tq_small_compress", "tq_small_dequant"):
        # decode-sized TurboQuant write / read (config 5 decode: the new tokens of a group of 32
        # sequences, 8 KV heads, into slot-mapped pool rows): K and V of 256 vectors each compressed
        # in one launch, 192 vectors read back
        n_tok = 32 if args.profile_kernel == "tq_small_compress" else 24
        rows = 256 * 1152
        rot = torch.from_numpy(K.tq_rotation_matrix(HD, 42)).to(dev)
        cen = torch.from_numpy(K.tq_codebook(HD, 4)[0]).to(dev)
        pool = torch.zeros((rows, NKV * 64), dtype=torch.uint8, device=dev)
        norms = torch.zeros((rows, NKV), dtype=torch.float16, device=dev)
        slots = (torch.randperm(256, generator=g, device=dev)[:n_tok].to(torch.int64) * 1152 + 1030).contiguous()
        x = torch.randn((n_tok, NKV, HD), generator=g, device=dev).to(torch.float16)
        K.tq_compress_slots(x, rot, cen, 4, pool, norms, slots)
        out = torch.empty_like(x)
        if args.profile_kernel == "tq_small_compress":
            xv = torch.randn((n_tok, NKV, HD), generator=g, device=dev).to(torch.float16)
            rot_v = torch.from_numpy(K.tq_rotation_matrix(HD, 542)).to(dev)
            pool_v, norms_v = torch.zeros_like(pool), torch.zeros_like(norms)
            fn = lambda: K.tq_compress_kv_slots(x, xv, rot, rot_v, cen, cen, 4, 4, pool, norms, pool_v, norms_v, slots)
        else:
            fn = lambda: K.tq_dequant_slots(pool, norms, rot, cen, 4, out, slots)
    else:
        tab = rnd(VOCAB, HID)
        ids = torch.randint(0, VOCAB, (T,), generator=g, device=dev, dtype=torch.int32)
        o = torch.empty((T, HID), device=dev, dtype=bf)
        fn = lambda: K.embedding(o, tab, ids)
    for _ in range(args.warmup):
        fn()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    fn()
    e1.record()
    torch.cuda.synchronize()
    print(json.dumps({"kernel": args.profile_kernel, "ms": round(e0.elapsed_time(e1), 4)}))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end (host buffers) measurement")
    ap.add_argument("--no-tq", action="store_true", help="skip the config-4 TurboQuant measurement")
    ap.add_argument("--no-decode", action="store_true", help="skip the config-2 decode-shaped measurement")
    ap.add_argument("--no-attention", action="store_true", help="skip the TurboQuant paged-attention measurement")
    ap.add_argument("--pipeline", action="store_true",
                    help="run config 5 (70B-shaped pipeline, NCCL stage handoff) at N=1 too (default: N > 1 only)")
    ap.add_argument("--no-pipeline", action="store_true", help="skip config 5")
    ap.add_argument("--only", default=None, choices=["tq", "decode", "attention"],
                    help="run only this workload on one GPU and print its figures")
    ap.add_argument("--profile-kernel", default=None, choices=["silu_mul", "add_rmsnorm", "rope", "embedding", "tq_compress",
                                                                   "tq_dequant", "tq_attention", "tq_attention_abi",
                                                                   "attention_fp16",
                                                                   "tq_small_compress", "tq_small_dequant"],
                    help="run only this kernel at its config-3 size (W warm-up launches + 1), for ncu captures")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.profile_kernel:
        profile_kernel(args)
        return
    if args.only:  # one workload on one GPU, printed alone (development runs; not the driver's line)
        fn = {"tq": lambda: run_tq_config4(args, 0, 1, local_rank), "decode": lambda: run_config2(args, local_rank),
              "attention": lambda: {"tq": run_tq_attention(args, local_rank),
                                    "tq_abi": run_tq_attention_abi(args, local_rank),
                                    "fp16": run_attention_fp16(args, local_rank)}}[args.only]
        print(json.dumps({"only": args.only, **fn()}), flush=True)
        return
    if args.impl == "reference":
        res = run_reference(args, rank)
        if res is not None:
            print(json.dumps(res), flush=True)
        return

    import datetime

    import torch
    import torch.distributed as dist

    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    res = run_ours(args, rank, world, local_rank)
    tq = None if args.no_tq else run_tq_config4(args, rank, world, local_rank)
    c5 = run_config5(args, rank, world, local_rank) if (args.pipeline or world > 1) and not args.no_pipeline \
        else None
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if res is not None and tq is not None:
        res["tq_config4"] = tq
    if res is not None and c5 is not None:
        res["pipeline_config5"] = c5
    if res is not None and world == 1 and not args.no_decode:
        res["decode_config2"] = run_config2(args, local_rank)
    if res is not None and world == 1 and not args.no_attention:
        res["tq_attention"] = run_tq_attention(args, local_rank)
        res["tq_attention_abi"] = run_tq_attention_abi(args, local_rank)
        res["attention_fp16"] = run_attention_fp16(args, local_rank)
    if res is not None:
        if world == 1 and not args.no_cpu_baseline:
            res["cpu_baseline"] = cpu_baseline(reps=3)
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
