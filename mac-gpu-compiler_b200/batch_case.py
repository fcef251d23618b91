"""A fixed batch-decode workload for profiler captures (ncu) of the batch step's kernels.

Loads the seeded random-init model (default: the Qwen3-0.6B geometry), prefills `--batch`
sequences of a `--prompt`-id prompt (one cache each), then runs `--steps` greedy batch steps with
qw_decode_batch (one captured graph replay per step: per layer the four skinny tcgen05 GEMMs, row
attention and merge, and the elementwise kernels; then the lm_head GEMM and the row argmax).
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
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--prompt", type=int, default=130)
    ap.add_argument("--steps", type=int, default=4)
    a = ap.parse_args()
    m = ci.CudaModel.load_model(randmodel.make_model(a.geometry, 0))
    caches, firsts = [], []
    for b in range(a.batch):
        c = ci.CudaKVCache(m, a.prompt + a.steps + 1)
        ids = randmodel.prompt_ids(a.prompt, m.config.vocab_size, seed=1 + b)
        m.prefill(ids[:-1], 0, c, logits=False)
        firsts.append(int(np.argmax(m.forward(ids[-1], a.prompt - 1, c))))
        caches.append(c)
    out = m.decode_batch(firsts, [a.prompt] * a.batch, a.steps, caches)
    print(f"{a.geometry}: batch {a.batch}, {a.steps} steps from position {a.prompt}; first row {out[0].tolist()}")


if __name__ == "__main__":
    main()
