"""Batch decode (qw_forward_batch / qw_decode_batch, the box workload's per-GPU batch variant)
against the CPU oracle, through the C ABI.

B independent sequences, each with its own prompt length and cache, step together. The rules are
the reference's parity rules applied per row (tests/metal_parity.rs:16-40): every row's logits
within 1e-2 of the oracle's forward() for that sequence (teacher-forced with the oracle's own
greedy tokens), and greedy tokens equal wherever the oracle's top-2 margin is at least 1e-2. The
batch's free-running decode must equal each row's own decode up to the first low-margin step.
"""
from __future__ import annotations

import numpy as np
import pytest

import cpu_oracle as co
import cuda_inference as ci
import randmodel

pytestmark = pytest.mark.gpu

TOL = 1e-2
MARGIN = 1e-2


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _rows(path, lens, seed0=11):
    """Oracle + GPU caches with row b's prompt (length lens[b]) already in; returns the oracle
    model, its caches, the GPU model, its caches and each row's next input token."""
    om = co.Model.load_model(path)
    gm = ci.CudaModel.load_model(path)
    ocs, gcs, nxt = [], [], []
    for b, n in enumerate(lens):
        ids = randmodel.prompt_ids(n, om.config.vocab_size, seed=seed0 + b)
        oc = co.KVCache(om)
        lg = None
        for p, t in enumerate(ids):
            lg = om.forward(t, p, oc)
        gc = ci.CudaKVCache(gm, n + 40)
        gm.prefill(ids, 0, gc, logits=False)
        ocs.append(oc)
        gcs.append(gc)
        nxt.append(co.argmax(lg))
    return om, ocs, gm, gcs, nxt


@pytest.mark.parametrize("geometry,lens,steps", [("tiny", [3, 17, 70, 129, 5], 6), ("mid", [9, 64, 65, 130], 4),
                                                  ("qwen3-0.6b", [6, 11, 4, 8, 7, 5, 9, 10], 2)])
def test_forward_batch_matches_oracle(geometry, lens, steps):
    om, ocs, gm, gcs, toks = _rows(randmodel.make_model(geometry, 0), lens)
    pos = list(lens)
    for _ in range(steps):
        got = gm.forward_batch(toks, pos, gcs)
        assert got.shape == (len(lens), om.config.vocab_size)
        nt = []
        for b in range(len(lens)):
            want = om.forward(toks[b], pos[b], ocs[b])
            assert np.isfinite(got[b]).all()
            assert np.abs(got[b] - want).max() <= TOL, (b, pos[b], float(np.abs(got[b] - want).max()))
            if co.top2_margin(want) >= MARGIN:
                assert co.argmax(got[b]) == co.argmax(want)
            nt.append(co.argmax(want))  # teacher-forced: the oracle's token goes in next
        toks, pos = nt, [p + 1 for p in pos]


def _oracle_greedy(om, oc, first, start, steps):
    """The oracle's greedy continuation and, per step, whether its top-2 margin was safe."""
    out, safe, t = [], [], first
    for i in range(steps):
        lg = om.forward(t, start + i, oc)
        t = co.argmax(lg)
        out.append(t)
        safe.append(co.top2_margin(lg) >= MARGIN)
    return out, safe


def test_decode_batch_matches_oracle_greedy(mid_model_path):
    lens = [5, 40, 64, 100, 7, 12]
    steps = 24
    om, ocs, gm, gcs, firsts = _rows(mid_model_path, lens)
    got = gm.decode_batch(firsts, lens, steps, gcs)
    assert got.shape == (len(lens), steps)
    for b in range(len(lens)):
        want, safe = _oracle_greedy(om, ocs[b], firsts[b], lens[b], steps)
        for i in range(steps):
            if not safe[i]:
                break  # after a low-margin step the sequences may legitimately diverge
            assert int(got[b, i]) == want[i], (b, i)


def test_decode_batch_equals_forward_batch_chain(mid_model_path):
    # the captured graph's on-device argmax chain equals forward_batch + host argmax, exactly
    lens = [8, 30, 61]
    _, _, gm, gc1, firsts = _rows(mid_model_path, lens)
    gc2 = [ci.CudaKVCache(gm, n + 40) for n in lens]
    for b, n in enumerate(lens):
        gm.prefill(randmodel.prompt_ids(n, gm.config.vocab_size, seed=11 + b), 0, gc2[b], logits=False)
    steps = 12
    got = gm.decode_batch(firsts, lens, steps, gc1)
    toks, pos = list(firsts), list(lens)
    for i in range(steps):
        lg = gm.forward_batch(toks, pos, gc2)
        toks = [co.argmax(lg[b]) for b in range(len(lens))]
        pos = [p + 1 for p in pos]
        assert [int(x) for x in got[:, i]] == toks, i


def test_decode_batch_is_deterministic_and_rows_independent(mid_model_path):
    lens = [10, 20, 30, 40]
    _, _, gm, gcs, firsts = _rows(mid_model_path, lens)
    a = gm.decode_batch(firsts, lens, 8, gcs)
    # the same rows again (fresh caches), alone and in a different batch order
    for order in ([0, 1, 2, 3], [3, 1, 0, 2]):
        cs = [ci.CudaKVCache(gm, n + 40) for n in lens]
        for b, n in enumerate(lens):
            gm.prefill(randmodel.prompt_ids(n, gm.config.vocab_size, seed=11 + b), 0, cs[b], logits=False)
        got = gm.decode_batch([firsts[i] for i in order], [lens[i] for i in order], 8, [cs[i] for i in order])
        for j, i in enumerate(order):
            assert (got[j] == a[i]).all(), (order, i)


def test_batch_limits_and_errors(tiny_model_path):
    gm = ci.CudaModel.load_model(tiny_model_path)
    cs = [ci.CudaKVCache(gm, 32) for _ in range(17)]
    for c in cs:
        gm.prefill([1, 2, 3], 0, c, logits=False)
    # 16 rows is the limit and works; 17 is refused
    out = gm.decode_batch([4] * 16, [3] * 16, 2, cs[:16])
    assert out.shape == (16, 2)
    with pytest.raises(ci.QwError) as e:
        gm.decode_batch([4] * 17, [3] * 17, 2, cs)
    assert e.value.code == ci.QW_ERR_ARG
    with pytest.raises(ci.QwError) as e:
        gm.decode_batch([4, 4], [3, 3], 2, [cs[0], cs[0]])          # the same cache twice
    assert e.value.code == ci.QW_ERR_ARG
    with pytest.raises(ci.QwError) as e:
        gm.decode_batch([4], [30], 5, [cs[0]])                      # runs past max_seq
    assert e.value.code == ci.QW_ERR_ARG
    with pytest.raises(ci.QwError) as e:
        gm.forward_batch([gm.config.vocab_size], [3], [cs[0]])      # token id out of range
    assert e.value.code == ci.QW_ERR_ARG
    other = ci.CudaModel.load_model(tiny_model_path)
    with pytest.raises(ci.QwError) as e:
        other.forward_batch([1], [3], [cs[0]])                       # a cache of another model
    assert e.value.code == ci.QW_ERR_ARG
