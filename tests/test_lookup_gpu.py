"""Prompt-lookup speculative decode (qw_decode_lookup) through the C ABI.

The reference's stated contract for speculation is "same greedy output with more than one token
per pass" (README.md:109-111). So the tokens must be the oracle's greedy continuation (up to the
first step whose oracle top-2 margin is below 1e-2, where float reordering may flip a token and
the sequences legitimately diverge), whatever the drafts were; and the pass count must drop when
the history repeats.
"""
from __future__ import annotations

import numpy as np
import pytest

import cpu_oracle as co
import cuda_inference as ci
import randmodel

pytestmark = pytest.mark.gpu
MARGIN = 1e-2


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _setup(path, prompt):
    om = co.Model.load_model(path)
    oc = co.KVCache(om)
    lg = None
    for p, t in enumerate(prompt):
        lg = om.forward(t, p, oc)
    gm = ci.CudaModel.load_model(path)
    return om, oc, gm, co.argmax(lg)


def _oracle_greedy(om, oc, first, start, steps):
    out, safe, t = [], [], first
    for i in range(steps):
        lg = om.forward(t, start + i, oc)
        t = co.argmax(lg)
        out.append(t)
        safe.append(co.top2_margin(lg) >= MARGIN)
    return out, safe


@pytest.mark.parametrize("repeat", [False, True])
def test_lookup_decode_is_greedy(mid_model_path, repeat):
    vocab = 10007
    base = randmodel.prompt_ids(24, vocab, seed=21)
    prompt = np.concatenate([base, base]) if repeat else randmodel.prompt_ids(48, vocab, seed=22)
    om, oc, gm, first = _setup(mid_model_path, prompt)
    steps = 40
    cache = ci.CudaKVCache(gm, len(prompt) + steps + 1)
    gm.prefill(prompt, 0, cache, logits=False)
    got, st = gm.decode_lookup(prompt, first, len(prompt), steps, cache, max_ngram=3, draft_max=7)
    assert len(got) == steps
    want, safe = _oracle_greedy(om, oc, first, len(prompt), steps)
    for i in range(steps):
        if not safe[i]:
            break
        assert got[i] == want[i], i
    assert st["accepted"] <= st["drafted"] and 1 <= st["passes"] <= steps
    # every pass emits its accepted drafts plus one token (the last pass may be cut short)
    assert st["passes"] + st["accepted"] >= steps


def test_lookup_on_the_full_geometry_saves_passes(full_model_path):
    # the random-init model's greedy output falls into repeats, which lookup drafts exactly
    prompt = randmodel.prompt_ids(16, 151936, seed=1)
    om, oc, gm, first = _setup(full_model_path, prompt)
    steps = 64
    cache = ci.CudaKVCache(gm, 100)
    gm.prefill(prompt, 0, cache, logits=False)
    got, st = gm.decode_lookup(prompt, first, len(prompt), steps, cache, max_ngram=3, draft_max=15)
    want, safe = _oracle_greedy(om, oc, first, len(prompt), steps)
    for i in range(steps):
        if not safe[i]:
            break
        assert got[i] == want[i], i
    assert st["passes"] < steps, st


def test_lookup_arguments(tiny_model_path):
    gm = ci.CudaModel.load_model(tiny_model_path)
    c = ci.CudaKVCache(gm, 16)
    gm.prefill([1, 2, 3], 0, c, logits=False)
    assert gm.decode_lookup([1, 2, 3], 4, 3, 0, c)[0] == []
    with pytest.raises(ci.QwError) as e:
        gm.decode_lookup([1, 2, 3], 4, 3, 20, c)                      # past max_seq
    assert e.value.code == ci.QW_ERR_ARG
    with pytest.raises(ci.QwError) as e:
        gm.decode_lookup([1, 2, 3], 4, 3, 4, c, draft_max=16)        # draft longer than the limit
    assert e.value.code == ci.QW_ERR_ARG
    with pytest.raises(ci.QwError) as e:
        gm.decode_lookup([1, 2, 3], 4, 3, 4, c, max_ngram=0)
    assert e.value.code == ci.QW_ERR_ARG
    # an empty context is allowed (drafts come from the output alone)
    toks, st = gm.decode_lookup([], 4, 3, 8, c)
    assert len(toks) == 8 and st["passes"] >= 1
