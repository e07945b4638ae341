#!/usr/bin/env python3
"""Extract the reference's committed fixture goldens into compact npz files.

Run once in a container that has the Fracture repository checked out (the GPU
box does not), e.g.::

    python tests/golden/make_golden.py --reference /path/to/Fracture

Inputs (read-only):

* ``tests/reference-fixture/prompt_{0,1}/`` — per-layer float32 dumps written by
  the reference's ``scripts/dump_reference.py`` on a CUDA GPU (torch 2.11).
* ``tests/fixtures/tiny-llama.gguf`` — the seeded tiny Llama whose weights
  produced those dumps (hidden 128, 4/2 heads, head_dim 32, inter 256,
  vocab 256, rope theta 5e5, eps 1e-5).

Output: ``tests/golden/fixture_prompt{0,1}.npz`` holding the tensors the
elementwise hot path consumes and produces (token ids, embedding table, norm
weights, and per layer the inputs/outputs of rmsnorm, residual add, rope and
silu_mul). Nothing is recomputed here; the values are the reference's own.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from oracle.refio import load_tensor  # noqa: E402

LAYER_FILES = [
    "input_hidden", "post_attn_norm", "q", "k", "q_rope", "k_rope", "attn_output",
    "post_attn_residual", "post_ffn_norm", "gate", "up", "silu_mul", "ffn_output",
    "output_hidden",
]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("FRACTURE_REFERENCE", str(HERE.parents[2] / "reference")),
                    help="the Fracture checkout (default: $FRACTURE_REFERENCE, or a checkout named `reference` "
                         "beside this repository)")
    ap.add_argument("--out", default=str(HERE))
    args = ap.parse_args()
    ref = Path(args.reference)

    from gguf import GGUFReader

    reader = GGUFReader(str(ref / "tests/fixtures/tiny-llama.gguf"))
    weights = {t.name: np.array(t.data) for t in reader.tensors}
    cfg = json.loads((ref / "tests/fixtures/tiny-llama.config.json").read_text())

    for p in (0, 1):
        pdir = ref / "tests/reference-fixture" / f"prompt_{p}"
        out: dict[str, np.ndarray] = {}
        out["token_ids"] = load_tensor(pdir / "token_ids.bin").astype(np.int32)
        if (pdir / "embeddings.bin").exists():
            out["embeddings"] = load_tensor(pdir / "embeddings.bin")[0]
        out["final_norm"] = load_tensor(pdir / "final_norm.bin")[0]
        out["token_embd"] = weights["token_embd.weight"].astype(np.float16)
        out["output_norm"] = weights["output_norm.weight"].astype(np.float16)
        for layer in range(cfg["num_layers"]):
            ldir = pdir / f"layer_{layer:02d}"
            out[f"l{layer}.attn_norm_w"] = weights[f"blk.{layer}.attn_norm.weight"].astype(np.float16)
            out[f"l{layer}.ffn_norm_w"] = weights[f"blk.{layer}.ffn_norm.weight"].astype(np.float16)
            for name in LAYER_FILES:
                f = ldir / f"{name}.bin"
                if not f.exists():
                    continue
                t = load_tensor(f)
                if t.ndim == 3 and t.shape[0] == 1:
                    t = t[0]
                out[f"l{layer}.{name}"] = t.astype(np.float32)
        meta = {k: cfg[k] for k in ("hidden_size", "num_q_heads", "num_kv_heads", "head_dim",
                                     "intermediate_size", "vocab_size", "rope_theta", "rms_norm_eps",
                                     "num_layers")}
        out["meta_json"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
        dst = Path(args.out) / f"fixture_prompt{p}.npz"
        np.savez_compressed(dst, **out)
        print(f"wrote {dst} ({dst.stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
