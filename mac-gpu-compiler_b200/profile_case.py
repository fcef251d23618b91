"""A small, fixed decode workload for profiler captures (ncu) of the decode kernel.

Loads the seeded random-init model (default: the full Qwen3-0.6B geometry, ~1.5 GB in HBM), runs
`--prompt` single-token forward() launches (positions 0..prompt-1) and then one `--decode`-step
greedy decode() launch. Every launch is qw::decode_kernel, so `ncu -k regex:decode_kernel -s S -c 1`
captures the forward launch at position S (S < prompt) or, with S == prompt, the decode launch.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

import numpy as np  # noqa: E402

import cuda_inference as ci  # noqa: E402
import randmodel  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--geometry", default="qwen3-0.6b", choices=sorted(randmodel.GEOMETRIES))
    ap.add_argument("--prompt", type=int, default=8)
    ap.add_argument("--decode", type=int, default=4)
    a = ap.parse_args()
    model = ci.CudaModel.load_model(randmodel.make_model(a.geometry, 0))
    cache = ci.CudaKVCache(model, a.prompt + a.decode + 1)
    ids = randmodel.prompt_ids(a.prompt, model.config.vocab_size, seed=1)
    logits = None
    for pos, tok in enumerate(ids):
        logits = model.forward(tok, pos, cache)
    toks = model.decode(int(np.argmax(logits)), a.prompt, a.decode, cache)
    print(f"{a.geometry}: {a.prompt} forward launches + 1 decode launch of {a.decode} steps -> {toks}")


if __name__ == "__main__":
    main()
