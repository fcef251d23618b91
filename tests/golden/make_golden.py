"""Generate the golden fixtures that pin the CPU oracle.

The reference's own golden vectors (tests/metal_parity.rs:13 "Paris" = 12095 after a 5-id
prompt; mlx_baseline/bench.py:48, the CPU engine's 16 greedy tokens) all require the real
Qwen3-0.6B checkpoint, which is not on these machines. So the oracle is pinned instead against an
independent implementation of the same architecture: Hugging Face ``transformers``'
``Qwen3ForCausalLM`` in float32 with eager attention, loaded from the very same seeded random-init
safetensors file (``randmodel.py``) and fed the same seeded token ids.

Fixtures written next to this script (float32 logits from transformers):
  hf_tiny.npz   tiny geometry, 8 positions, full logits
  hf_mid.npz    Qwen3-0.6B per-layer shapes with 3 layers, 4 positions, full logits
  hf_full.npz   the full Qwen3-0.6B geometry, 3 positions: top-16 ids/values and 512 logits at
                fixed seeded indices (full rows would be 1.8 MB)
  hf_*_long.npz longer prompts in the same sampled form (top-16 and 256 sampled logits per
                position, plus the top-2 margin): tiny 128, mid 48 and full 24 positions, so the
                RoPE table and the attention softmax are pinned over longer contexts

Run from the repo root:  python tests/golden/make_golden.py
This script needs ``transformers`` (importable in the build container); the tests that read the
fixtures need only numpy and the oracle.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "mac-gpu-compiler_b200"))
import randmodel  # noqa: E402

SPECS = {"tiny": 8, "mid": 4, "qwen3-0.6b": 3}
N_SAMPLE = 512
TOPK = 16


def hf_logits(geometry: str, ids: list[int]) -> np.ndarray:
    from safetensors.torch import load_file
    from transformers import Qwen3Config, Qwen3ForCausalLM

    path = randmodel.make_model(geometry, 0)
    cfgd = json.loads((path.parent / "config.json").read_text())
    cfg = Qwen3Config(**{k: v for k, v in cfgd.items() if k not in ("architectures", "torch_dtype")})
    cfg._attn_implementation = "eager"
    model = Qwen3ForCausalLM(cfg).float().eval()
    sd = {k: v.float() for k, v in load_file(str(path)).items()}
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not missing and not unexpected, (missing, unexpected)
    with torch.no_grad():
        return model(torch.tensor([ids])).logits[0].float().numpy()


def main() -> None:
    torch.set_num_threads(8)
    for geometry, n in SPECS.items():
        vocab = randmodel.GEOMETRIES[geometry]["vocab_size"]
        ids = randmodel.prompt_ids(n, vocab, seed=1)
        logits = hf_logits(geometry, ids)
        if geometry == "qwen3-0.6b":
            rng = np.random.Generator(np.random.PCG64(7))
            idx = np.sort(rng.choice(vocab, N_SAMPLE, replace=False)).astype(np.int64)
            top_ids = np.argsort(-logits, axis=1, kind="stable")[:, :TOPK].astype(np.int64)
            np.savez(HERE / "hf_full.npz", ids=np.array(ids, np.int64), sample_idx=idx,
                     sample_logits=logits[:, idx].astype(np.float32), top_ids=top_ids,
                     top_logits=np.take_along_axis(logits, top_ids, 1).astype(np.float32),
                     argmax=logits.argmax(1).astype(np.int64))
            print(geometry, "->", HERE / "hf_full.npz")
        else:
            name = "hf_" + geometry + ".npz"
            np.savez(HERE / name, ids=np.array(ids, np.int64), logits=logits.astype(np.float32))
            print(geometry, "->", HERE / name)


LONG_SPECS = {"tiny": 128, "mid": 48, "qwen3-0.6b": 24}
N_SAMPLE_LONG = 256


def main_long() -> None:
    torch.set_num_threads(8)
    for geometry, n in LONG_SPECS.items():
        vocab = randmodel.GEOMETRIES[geometry]["vocab_size"]
        ids = randmodel.prompt_ids(n, vocab, seed=2)
        logits = hf_logits(geometry, ids)
        rng = np.random.Generator(np.random.PCG64(11))
        idx = np.sort(rng.choice(vocab, min(N_SAMPLE_LONG, vocab), replace=False)).astype(np.int64)
        top_ids = np.argsort(-logits, axis=1, kind="stable")[:, :TOPK].astype(np.int64)
        top = np.take_along_axis(logits, top_ids, 1).astype(np.float32)
        name = "hf_" + ("full" if geometry == "qwen3-0.6b" else geometry) + "_long.npz"
        np.savez(HERE / name, ids=np.array(ids, np.int64), sample_idx=idx, sample_logits=logits[:, idx].astype(np.float32),
                 top_ids=top_ids, top_logits=top, argmax=logits.argmax(1).astype(np.int64),
                 margin=(top[:, 0] - top[:, 1]).astype(np.float32))
        print(geometry, "->", HERE / name)


if __name__ == "__main__":
    main()
    main_long()
