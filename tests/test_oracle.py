"""The CPU oracle (restatement of metal_infrence_engine/src/cpu_inference.rs) against golden
fixtures from transformers' Qwen3 on the same seeded weights, plus the reference's own rules
(argmax tie rule, bytes-per-token rule)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import cpu_oracle as co

GOLDEN = Path(__file__).resolve().parent / "golden"
# float32 implementations with different summation orders agree to ~1e-6 here; the bound is
# two orders of magnitude below the engine parity bar (1e-2)
HF_TOL = 1e-4


@pytest.mark.parametrize("geometry,fixture", [("tiny", "hf_tiny.npz"), ("mid", "hf_mid.npz")])
def test_oracle_matches_transformers(geometry, fixture, request):
    path = request.getfixturevalue(f"{geometry}_model_path")
    d = np.load(GOLDEN / fixture)
    m = co.Model.load_model(path)
    cache = co.KVCache(m)
    for pos, tok in enumerate(d["ids"]):
        lg = m.forward(int(tok), pos, cache)
        assert np.isfinite(lg).all()
        assert np.abs(lg - d["logits"][pos]).max() < HF_TOL, pos
        assert co.argmax(lg) == int(np.argmax(d["logits"][pos]))
    assert len(cache) == len(d["ids"])


def test_oracle_matches_transformers_full_geometry(full_model_path):
    d = np.load(GOLDEN / "hf_full.npz")
    m = co.Model.load_model(full_model_path)
    cache = co.KVCache(m)
    for pos, tok in enumerate(d["ids"]):
        lg = m.forward(int(tok), pos, cache)
        assert np.abs(lg[d["sample_idx"]] - d["sample_logits"][pos]).max() < HF_TOL
        assert np.abs(lg[d["top_ids"][pos]] - d["top_logits"][pos]).max() < HF_TOL
        assert co.argmax(lg) == int(d["argmax"][pos])


@pytest.mark.parametrize("geometry,fixture", [("tiny", "hf_tiny_long.npz"), ("mid", "hf_mid_long.npz"),
                                              ("full", "hf_full_long.npz")])
def test_oracle_matches_transformers_longer_prompts(geometry, fixture, request):
    """Longer prompts (128, 48 and 24 positions): the oracle's per-position logits against
    transformers' at 256 sampled vocabulary ids and the top 16, and the same argmax wherever
    transformers' top-2 margin leaves room for the tolerance."""
    path = request.getfixturevalue(f"{geometry}_model_path")
    d = np.load(GOLDEN / fixture)
    m = co.Model.load_model(path)
    cache = co.KVCache(m)
    for pos, tok in enumerate(d["ids"]):
        lg = m.forward(int(tok), pos, cache)
        assert np.abs(lg[d["sample_idx"]] - d["sample_logits"][pos]).max() < HF_TOL, pos
        assert np.abs(lg[d["top_ids"][pos]] - d["top_logits"][pos]).max() < HF_TOL, pos
        if d["margin"][pos] > 2 * HF_TOL:
            assert co.argmax(lg) == int(d["argmax"][pos]), pos


def test_weight_bytes_rule_matches_reference(full_model_path):
    # tests/mbu.rs:19-30 on the Qwen3-0.6B geometry gives the reference's published
    # 1,192,101,888 B/token (mlx_baseline/results/engine_metal_m1_ai.json:140)
    m = co.Model.load_model(full_model_path)
    assert m.weight_bytes_per_token() == 1_192_101_888


def test_argmax_first_strict_max_rule():
    # tests/common/mod.rs:17-22: ties go to the lowest index; a NaN at index 0 sticks
    assert co.argmax(np.array([1, 3, 3, 2], np.float32)) == 1
    assert co.argmax(np.array([np.nan, 5, 7], np.float32)) == 0
    assert co.argmax(np.array([1, np.nan, 7], np.float32)) == 2
    assert co.argmax(np.array([-np.inf, -np.inf], np.float32)) == 0


def test_cache_layout_and_growth(tiny_model_path):
    m = co.Model.load_model(tiny_model_path)
    c = m.config
    cache = co.KVCache(m)
    for pos, tok in enumerate([1, 2, 3]):
        m.forward(tok, pos, cache)
    k, v = cache.layer(0)
    assert k.shape == (3, c.num_key_value_heads * c.head_dim) and v.shape == k.shape
    # pos past the cache length is an error (the reference panics on the out-of-range slice)
    with pytest.raises(RuntimeError):
        m.forward(4, 7, cache)


def test_oracle_load_errors(tmp_path):
    with pytest.raises(OSError):
        co.Model.load_model(tmp_path / "missing.safetensors")
    bad = tmp_path / "model.safetensors"
    bad.write_bytes(b"\x10\x00\x00\x00\x00\x00\x00\x00{not json}      ")
    (tmp_path / "config.json").write_text("{}")
    with pytest.raises(OSError):
        co.Model.load_model(bad)


@pytest.mark.parametrize("geometry,n,start", [("tiny", 37, 0), ("tiny", 20, 9), ("mid", 6, 0)])
def test_forward_seq_is_bit_identical_to_token_by_token(geometry, n, start, request):
    """The layer-major multi-position forward (used to get long-prompt oracle references in
    seconds) must reproduce the token-by-token loop exactly: logits and cache, bit for bit."""
    path = request.getfixturevalue(f"{geometry}_model_path")
    m = co.Model.load_model(path)
    import randmodel
    ids = randmodel.prompt_ids(start + n, m.config.vocab_size, seed=4)
    c1, c2 = co.KVCache(m), co.KVCache(m)
    want = [m.forward(t, p, c1) for p, t in enumerate(ids)]
    if start:
        m.forward_seq(ids[:start], 0, c2, out_positions=[])
    pick = list(range(0, n, 3)) + [n - 1]
    got = m.forward_seq(ids[start:], start, c2, out_positions=pick)
    for row, i in enumerate(pick):
        assert np.array_equal(got[row], want[start + i]), i
    for l in range(m.config.num_hidden_layers):
        k1, v1 = c1.layer(l)
        k2, v2 = c2.layer(l)
        assert np.array_equal(k1, k2) and np.array_equal(v1, v2)
    with pytest.raises(RuntimeError):      # the cache must hold exactly start_pos positions
        m.forward_seq(ids[:2], 3, c2)
