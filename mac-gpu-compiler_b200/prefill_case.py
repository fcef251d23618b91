"""A fixed batched-prefill workload for profiler captures (ncu) of the prefill's kernels.

Loads the seeded random-init model (default: the Qwen3-0.6B geometry), then runs `--passes`
prefill passes over a `--prompt`-id prompt with device-resident ids and logits. Each pass launches,
per layer, the four tcgen05 GEMMs (q|k|v, o, gate|up, down) and the elementwise kernels around them,
then the lm_head GEMM.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

import torch  # noqa: E402

import cuda_inference as ci  # noqa: E402
import randmodel  # noqa: E402


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--geometry", default="qwen3-0.6b", choices=sorted(randmodel.GEOMETRIES))
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--passes", type=int, default=2)
    a = ap.parse_args()
    m = ci.CudaModel.load_model(randmodel.make_model(a.geometry, 0))
    cache = ci.CudaKVCache(m, a.prompt + 1)
    ids = torch.tensor(randmodel.prompt_ids(a.prompt, m.config.vocab_size, seed=1), dtype=torch.int32, device="cuda")
    logits = torch.empty(a.prompt, m.config.vocab_size, device="cuda")
    for _ in range(a.passes):
        m.prefill_device(cache, ids.data_ptr(), a.prompt, 0, logits.data_ptr())
    m.sync()
    print(f"{a.geometry}: {a.passes} prefill passes of {a.prompt} tokens; last argmax {int(logits[-1].argmax())}")


if __name__ == "__main__":
    main()
