#!/usr/bin/env python3
"""Regenerate the golden fixtures under ``tests/golden/``.

1. ``ref_parity_small.json``: the reference's own fixture generator
   (``scripts/generate_parity_fixture.py`` of arkavo-ai/WeDLM-rs, numpy only) is run
   from the reference checkout into a temporary file; the output is checked to
   equal the reference's committed fixture ``tests/fixtures/wedlm_parity_small.json``
   (all numbers within 1e-7) and saved here.  It pins ``forward_with_positions`` with
   explicit non-contiguous positions ``[0, 2, 5]`` (1 layer, f32).

2. ``c1_streaming.json``: the tiny fp32 workload (2 layers, hidden 256, 4/2 heads,
   head_dim 64, ffn 768, vocab 4096, 32-token prompt, one 16-slot block) run through
   the oracle: per-step reordered ids/positions, entropies, selections, committed
   ids.  It is a regression record for the CUDA path, produced by the oracle.

Usage: ``python tests/golden/make_golden.py [--reference /path/to/WeDLM-rs]`` (or set
``WEDLM_REFERENCE``).
Needs the reference checkout only for (1).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))


def make_ref_fixture(reference: Path) -> None:
    gen = reference / "scripts" / "generate_parity_fixture.py"
    committed = reference / "tests" / "fixtures" / "wedlm_parity_small.json"
    with tempfile.TemporaryDirectory() as td:
        out = Path(td) / "fixture.json"
        subprocess.run([sys.executable, str(gen), "--output", str(out)], check=True,
                       cwd=td, stdout=subprocess.DEVNULL)
        fresh = json.loads(out.read_text())
    ref = json.loads(committed.read_text())

    def close(a, b):
        if isinstance(a, dict):
            return a.keys() == b.keys() and all(close(a[k], b[k]) for k in a)
        if isinstance(a, list):
            return len(a) == len(b) and all(close(x, y) for x, y in zip(a, b))
        if isinstance(a, float) or isinstance(b, float):
            return abs(float(a) - float(b)) <= 1e-7
        return a == b

    assert close(fresh, ref), "regenerated fixture differs from the reference's committed fixture"
    (HERE / "ref_parity_small.json").write_text(json.dumps(fresh, sort_keys=True) + "\n")
    print("wrote ref_parity_small.json")


def c1_config():
    from oracle.model import WeDLMConfig
    return WeDLMConfig(vocab_size=4096, hidden_size=256, num_hidden_layers=2,
                       num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                       intermediate_size=768, max_position_embeddings=256,
                       rope_theta=1_000_000.0, rms_norm_eps=1e-6, qk_norm=True,
                       eos_token_id=0, mask_token_id=4095, dtype="float32")


def make_c1() -> None:
    from oracle.model import OracleModel, random_weights
    from oracle.decoder import OracleDecoder
    from oracle.sampler import SamplingParams
    cfg = c1_config()
    w = random_weights(cfg, seed=0, std=0.02)
    m = OracleModel(cfg, w, "f32")
    prompt = np.random.default_rng(0).integers(1, 4095, size=32).tolist()
    params = SamplingParams(temperature=0.0, entropy_threshold=0.8, distance_penalty=0.05,
                            max_tokens_per_step=8)
    dec = OracleDecoder(m, cfg.mask_token_id, cfg.eos_token_id)
    ids, stats = dec.generate_streaming(prompt, 16, 16, params)
    rec = {
        "config": cfg.to_dict(), "seed": 0, "std": 0.02, "prompt": prompt,
        "max_new_tokens": 16, "window": 16,
        "params": {"temperature": 0.0, "tau": 0.8, "lambda": 0.05, "cap": 8},
        "output_ids": ids, "steps": stats.steps,
        "trace": [{"n_commit": t.n_commit, "reordered_tokens": t.reordered_tokens,
                   "reordered_positions": t.reordered_positions, "num_filled": t.num_filled,
                   "entropies": [float(x) for x in t.entropies], "effective_max": t.effective_max,
                   "selected": t.selected, "sampled": t.sampled} for t in dec.trace],
    }
    (HERE / "c1_streaming.json").write_text(json.dumps(rec) + "\n")
    print("wrote c1_streaming.json", "steps", stats.steps)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("WEDLM_REFERENCE"),
                    help="WeDLM-rs checkout (default: $WEDLM_REFERENCE)")
    a = ap.parse_args()
    ref = Path(a.reference) if a.reference else None
    if ref is not None and (ref / "scripts" / "generate_parity_fixture.py").exists():
        make_ref_fixture(ref)
    else:
        print("reference checkout not found; keeping the committed ref_parity_small.json")
    make_c1()


if __name__ == "__main__":
    main()
