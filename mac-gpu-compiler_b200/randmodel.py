"""Seeded random-init Qwen3 model directories (safetensors + config.json).

There is no network and no real checkpoint on these machines, so every test and benchmark runs on
a synthetic model with the exact Qwen3-0.6B tensor names, shapes and dtype (bf16) that the
reference engine loads (metal_infrence_engine/src/cpu_inference.rs:58-96, :109-177). The file is
written by ``csrc/randmodel.cpp`` (built into ``librandmodel.so``); this module adds
``config.json`` with the ten fields the reference reads (cpu_inference.rs:21-33) plus the
Hugging Face keys needed to load the same directory with ``transformers``.

Named geometries:
  qwen3-0.6b  the benchmark model: hidden 1024, 28 layers, 16/8 heads, head_dim 128,
              SwiGLU 3072, vocab 151936, tied embedding, RoPE theta 1e6, eps 1e-6
  mid         the same per-layer shapes with 3 layers and a ragged vocab (10007)
  tiny        a small model for fast CPU checks (hidden 256, 2 layers, vocab 1000)
"""
from __future__ import annotations

import ctypes
import json
import os
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent

GEOMETRIES = {
    "qwen3-0.6b": dict(hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                       num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                       vocab_size=151936),
    "mid": dict(hidden_size=1024, intermediate_size=3072, num_hidden_layers=3,
                num_attention_heads=16, num_key_value_heads=8, head_dim=128, vocab_size=10007),
    "tiny": dict(hidden_size=256, intermediate_size=768, num_hidden_layers=2,
                 num_attention_heads=4, num_key_value_heads=2, head_dim=128, vocab_size=1000),
}

RMS_NORM_EPS = 1e-6
ROPE_THETA = 1e6
EOS_TOKEN_ID = 151645


def _lib():
    path = _HERE / "librandmodel.so"
    if not path.exists():
        raise RuntimeError(f"{path} is missing: run `python {_HERE / 'build.py'}` first")
    lib = ctypes.CDLL(str(path))
    lib.rm_write_model.restype = ctypes.c_int
    lib.rm_write_model.argtypes = [ctypes.c_char_p] + [ctypes.c_uint32] * 7 + [ctypes.c_uint64, ctypes.c_int]
    return lib


def config_dict(geometry: str) -> dict:
    g = GEOMETRIES[geometry]
    cfg = dict(g)
    cfg.update(rms_norm_eps=RMS_NORM_EPS, rope_theta=ROPE_THETA, eos_token_id=EOS_TOKEN_ID,
               bos_token_id=151643, model_type="qwen3", architectures=["Qwen3ForCausalLM"],
               tie_word_embeddings=True, hidden_act="silu", attention_bias=False,
               max_position_embeddings=40960, torch_dtype="bfloat16")
    return cfg


def default_root() -> Path:
    return Path(os.environ.get("QW_MODEL_CACHE", "/tmp/qw_models"))


def make_model(geometry: str = "qwen3-0.6b", seed: int = 0, root: Path | None = None) -> Path:
    """Return the path of ``<root>/<geometry>-s<seed>/model.safetensors``, writing it if absent."""
    root = Path(root) if root is not None else default_root()
    d = root / f"{geometry}-s{seed}"
    st = d / "model.safetensors"
    cfg_path = d / "config.json"
    cfg = config_dict(geometry)
    if st.exists() and cfg_path.exists():
        try:
            if json.loads(cfg_path.read_text()) == cfg:
                return st
        except ValueError:
            pass
    d.mkdir(parents=True, exist_ok=True)
    tmp = d / f"model.safetensors.tmp{os.getpid()}"
    g = GEOMETRIES[geometry]
    rc = _lib().rm_write_model(str(tmp).encode(), g["hidden_size"], g["intermediate_size"],
                               g["num_hidden_layers"], g["num_attention_heads"],
                               g["num_key_value_heads"], g["head_dim"], g["vocab_size"], seed, 0)
    if rc != 0:
        raise RuntimeError(f"writing {tmp} failed")
    os.replace(tmp, st)
    cfg_path.write_text(json.dumps(cfg, indent=1))
    return st


def prompt_ids(n: int, vocab: int, seed: int = 1) -> list[int]:
    """n token ids uniform in [0, vocab) from `seed` (stand-in for the reference's 130-id `ai` prompt)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    return [int(t) for t in rng.integers(0, vocab, size=n)]


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--geometry", default="qwen3-0.6b", choices=sorted(GEOMETRIES))
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--root", default=None)
    a = ap.parse_args()
    print(make_model(a.geometry, a.seed, a.root))
