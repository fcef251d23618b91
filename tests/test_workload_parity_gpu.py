"""GPU parity on the full Qwen3-0.6B geometry for the workloads the benchmark measures.

The rules are the reference's tests/metal_parity.rs:16-40 (logits finite and within 1e-2 max-abs of
the CPU engine at every checked position; the same greedy token unless the CPU's top-2 logit
margin is below 1e-2) and :44-71 (the pipelined greedy decode gives the CPU's greedy tokens). The
CPU side is the oracle (C++ restatement of cpu_inference.rs); its prompts are run with
``forward_seq``, which is bit-identical to token-by-token ``forward`` (tests/test_oracle.py), so a
2048-position reference costs seconds.

  * 130-id prompt fed token by token, then 128 greedy steps (positions 0..257): logits at every
    one of the 258 positions, teacher-forced with the oracle's tokens; the free-running qw_decode
    tokens against the oracle's greedy chain up to its first low-margin step.
  * 2048-id prompt fed token by token, then 32 greedy steps (the long-context workload's split-K
    attention over 2048+ positions): logits at sampled prompt positions and every decode position;
    the free-running decode against the oracle's chain.
  * one 512-token qw_prefill: every position's logits and the K/V cache against the oracle's
    token-by-token prefill; then 64 greedy decode steps from the prefilled cache.
"""
from __future__ import annotations

import numpy as np
import pytest

import cpu_oracle as co
import cuda_inference as ci
import randmodel

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

MAX_ABS_DIFF = 1e-2   # metal_parity.rs:14
MARGIN = 1e-2         # greedy tokens must agree where the oracle's top-2 gap is at least this
KV_TOL = 1e-3


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.fixture(scope="module")
def models(full_model_path):
    cpu = co.Model.load_model(full_model_path)
    gpu = ci.CudaModel.load_model(full_model_path)
    yield cpu, gpu
    gpu.close()


def _check(pos, want, got, label):
    assert np.isfinite(got).all(), f"{label} pos {pos}: non-finite logits"
    d = float(np.abs(want - got).max())
    assert d < MAX_ABS_DIFF, f"{label} pos {pos}: logits differ by {d}"
    if co.top2_margin(want) >= MARGIN:
        assert co.argmax(want) == co.argmax(got), f"{label} pos {pos}: different greedy token"
    return d


def _oracle_chain(cpu, cache, first, start, steps):
    """The oracle's free-running greedy continuation: (tokens, logits of each step, margins)."""
    toks, logits, tok = [], [], first
    for i in range(steps):
        lg = cpu.forward(tok, start + i, cache)
        tok = co.argmax(lg)
        toks.append(tok)
        logits.append(lg)
    return toks, logits


def _agree_until_low_margin(got, want, logits):
    """got == want up to (and including) the first step whose oracle margin is below MARGIN."""
    for i, (g, w) in enumerate(zip(got, want)):
        if co.top2_margin(logits[i]) < MARGIN:
            return i
        assert g == w, f"step {i}: gpu {g} != oracle {w}"
    return len(want)


@pytest.fixture(scope="module")
def ref130(models):
    """The oracle's side of the 130 + 128 workload, computed once for both decode kernels."""
    cpu, _ = models
    n_prompt, n_dec = 130, 128
    ids = randmodel.prompt_ids(n_prompt, cpu.config.vocab_size, seed=1)
    oc = co.KVCache(cpu)
    want_prompt = cpu.forward_seq(ids, 0, oc)
    first = co.argmax(want_prompt[-1])
    want_toks, want_dec = _oracle_chain(cpu, oc, first, n_prompt, n_dec)
    last = cpu.config.num_hidden_layers - 1
    return dict(ids=ids, want_prompt=want_prompt, first=first, want_toks=want_toks, want_dec=want_dec,
                kv={l: oc.layer(l) for l in (0, last)})


@pytest.mark.parametrize("decoder", ["grid", "cluster"])
def test_decode_workload_130_plus_128_every_position(models, ref130, decoder, full_model_path, monkeypatch):
    cpu, gpu = models
    if decoder == "cluster":
        monkeypatch.setenv("QW_DECODER", "cluster")
        gpu = ci.CudaModel.load_model(full_model_path)
    assert gpu.decoder_kind == decoder
    ids, first = ref130["ids"], ref130["first"]
    want_prompt, want_toks, want_dec = ref130["want_prompt"], ref130["want_toks"], ref130["want_dec"]
    n_prompt, n_dec = len(ids), len(want_toks)

    # teacher-forced: the GPU is fed the oracle's tokens, logits compared at all 258 positions
    gc = ci.CudaKVCache(gpu, n_prompt + n_dec + 1)
    worst = 0.0
    for pos, tok in enumerate(ids):
        worst = max(worst, _check(pos, want_prompt[pos], gpu.forward(tok, pos, gc), "prompt"))
    fed = [first] + want_toks[:-1]
    for i, tok in enumerate(fed):
        worst = max(worst, _check(n_prompt + i, want_dec[i], gpu.forward(tok, n_prompt + i, gc), "decode"))
    # KV cache of the whole sequence against the oracle's (first and last layer)
    for l, (ko, vo) in ref130["kv"].items():
        kg, vg = gc.layer(l, n_prompt + n_dec)
        assert np.abs(kg - ko).max() < KV_TOL and np.abs(vg - vo).max() < KV_TOL, l

    # free-running: one qw_decode launch of 128 steps from a forward-filled prompt cache
    fc = ci.CudaKVCache(gpu, n_prompt + n_dec + 1)
    for pos, tok in enumerate(ids):
        gpu.forward(tok, pos, fc)
    got = gpu.decode(first, n_prompt, n_dec, fc)
    agreed = _agree_until_low_margin(got, want_toks, want_dec)
    print(f"130+128 ({decoder}): max |cpu - gpu| = {worst:.3e} over 258 positions; decode agrees for {agreed} steps")


def test_long_context_2048_plus_32(models):
    cpu, gpu = models
    n_prompt, n_dec = 2048, 32
    ids = randmodel.prompt_ids(n_prompt, cpu.config.vocab_size, seed=2)
    check = sorted(set(range(0, n_prompt, 97)) | {1023, 1024, n_prompt - 2, n_prompt - 1})
    oc = co.KVCache(cpu)
    want_prompt = dict(zip(check, cpu.forward_seq(ids, 0, oc, out_positions=check)))
    first = co.argmax(want_prompt[n_prompt - 1])
    want_toks, want_dec = _oracle_chain(cpu, oc, first, n_prompt, n_dec)

    gc = ci.CudaKVCache(gpu, n_prompt + n_dec + 1)
    worst = 0.0
    for pos, tok in enumerate(ids):
        lg = gpu.forward(tok, pos, gc)
        if pos in want_prompt:
            worst = max(worst, _check(pos, want_prompt[pos], lg, "prompt"))
    snapshot = [gc.layer(l, n_prompt) for l in (0, cpu.config.num_hidden_layers - 1)]
    fed = [first] + want_toks[:-1]
    for i, tok in enumerate(fed):
        worst = max(worst, _check(n_prompt + i, want_dec[i], gpu.forward(tok, n_prompt + i, gc), "decode"))
    for (kg, vg), l in zip(snapshot, (0, cpu.config.num_hidden_layers - 1)):
        ko, vo = oc.layer(l)
        assert np.abs(kg - ko[:n_prompt]).max() < KV_TOL and np.abs(vg - vo[:n_prompt]).max() < KV_TOL, l

    # free-running decode over the same prompt cache (positions 2048.. are rewritten)
    got = gpu.decode(first, n_prompt, n_dec, gc)
    agreed = _agree_until_low_margin(got, want_toks, want_dec)
    print(f"2048+32: max |cpu - gpu| = {worst:.3e}; decode agrees for {agreed} steps")


def test_prefill_512_then_64_decode(models):
    cpu, gpu = models
    n, n_dec = 512, 64
    ids = randmodel.prompt_ids(n, cpu.config.vocab_size, seed=3)
    oc = co.KVCache(cpu)
    want = cpu.forward_seq(ids, 0, oc)
    gc = ci.CudaKVCache(gpu, n + n_dec + 1)
    got = gpu.prefill(ids, 0, gc)
    assert got.shape == want.shape and np.isfinite(got).all()
    diff = np.abs(got - want).max(axis=1)
    assert float(diff.max()) <= MAX_ABS_DIFF, f"pos {int(diff.argmax())}: {float(diff.max())}"
    for pos in range(n):
        if co.top2_margin(want[pos]) >= MARGIN:
            assert co.argmax(want[pos]) == co.argmax(got[pos]), pos
    for l in range(cpu.config.num_hidden_layers):
        kg, vg = gc.layer(l, n)
        ko, vo = oc.layer(l)
        assert np.abs(kg - ko).max() < KV_TOL and np.abs(vg - vo).max() < KV_TOL, l
    first = co.argmax(want[-1])
    want_toks, want_dec = _oracle_chain(cpu, oc, first, n, n_dec)
    got_toks = gpu.decode(first, n, n_dec, gc)
    agreed = _agree_until_low_margin(got_toks, want_toks, want_dec)
    print(f"prefill 512: max |cpu - gpu| = {float(diff.max()):.3e}; decode agrees for {agreed} steps")
