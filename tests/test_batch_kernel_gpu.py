"""The persistent batch decode kernel (QW_BATCH_DECODER=persistent: qw_decode_batch for at most 8
rows in one launch) against the CPU oracle, through the C ABI.

The rules are the batch tests' (the reference's parity rules per row, tests/metal_parity.rs:16-40):
greedy tokens equal to the oracle's wherever its top-2 margin is at least 1e-2, the K/V written
for every decoded position within 1e-3 of the oracle's cache, and the same tokens as the row-mode
path up to the first low-margin step.
"""
from __future__ import annotations

import numpy as np
import pytest

import cpu_oracle as co
import cuda_inference as ci
import randmodel

pytestmark = pytest.mark.gpu

MARGIN = 1e-2
KV_TOL = 1e-3


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _load(path, monkeypatch, persistent=True):
    if persistent:
        monkeypatch.setenv("QW_BATCH_DECODER", "persistent")
    else:
        monkeypatch.delenv("QW_BATCH_DECODER", raising=False)
    return ci.CudaModel.load_model(path)


def _prefilled(gm, om, lens, extra, seed0=11):
    gcs, ocs, firsts = [], [], []
    for b, n in enumerate(lens):
        ids = randmodel.prompt_ids(n, gm.config.vocab_size, seed=seed0 + b)
        gc = ci.CudaKVCache(gm, n + extra)
        gm.prefill(ids, 0, gc, logits=False)
        gcs.append(gc)
        if om is not None:
            oc = co.KVCache(om)
            lg = None
            for p, t in enumerate(ids):
                lg = om.forward(t, p, oc)
            ocs.append(oc)
            firsts.append(co.argmax(lg))
    return gcs, ocs, firsts


def _oracle_greedy(om, oc, first, start, steps):
    toks, safe, t = [], [], first
    for i in range(steps):
        lg = om.forward(t, start + i, oc)
        t = co.argmax(lg)
        toks.append(t)
        safe.append(co.top2_margin(lg) >= MARGIN)
    return toks, safe


@pytest.mark.parametrize("lens", [[5, 40, 64, 100, 7, 12], [33], [9, 130, 2, 77, 50, 64, 18, 3]])
def test_persistent_batch_matches_oracle_greedy(mid_model_path, monkeypatch, lens):
    om = co.Model.load_model(mid_model_path)
    gm = _load(mid_model_path, monkeypatch)
    assert gm.batch_decoder_kind == "persistent"
    steps = 20
    gcs, ocs, firsts = _prefilled(gm, om, lens, steps + 4)
    got = gm.decode_batch(firsts, lens, steps, gcs)
    assert got.shape == (len(lens), steps)
    for b in range(len(lens)):
        want, safe = _oracle_greedy(om, ocs[b], firsts[b], lens[b], steps)
        for i in range(steps):
            if not safe[i]:
                break
            assert int(got[b, i]) == want[i], (b, i)
        # every position the launch decoded wrote K and V like the oracle (before the first low-margin step)
        n_ok = lens[b] + (next((i for i in range(steps) if not safe[i]), steps))
        for layer in range(gm.config.num_hidden_layers):
            k, v = gcs[b].layer(layer, n_ok)
            ok_, ov_ = ocs[b].layer(layer)
            assert float(np.abs(k[lens[b]:n_ok] - ok_[lens[b]:n_ok]).max(initial=0.0)) < KV_TOL
            assert float(np.abs(v[lens[b]:n_ok] - ov_[lens[b]:n_ok]).max(initial=0.0)) < KV_TOL


def test_persistent_batch_full_geometry(full_model_path, monkeypatch):
    om = co.Model.load_model(full_model_path)
    gm = _load(full_model_path, monkeypatch)
    assert gm.batch_decoder_kind == "persistent"
    lens = [6, 11, 4, 8, 7, 5, 9, 10]
    steps = 6
    gcs, ocs, firsts = _prefilled(gm, om, lens, steps + 2)
    got = gm.decode_batch(firsts, lens, steps, gcs)
    for b in range(len(lens)):
        want, safe = _oracle_greedy(om, ocs[b], firsts[b], lens[b], steps)
        for i in range(steps):
            if not safe[i]:
                break
            assert int(got[b, i]) == want[i], (b, i)


def test_persistent_and_row_mode_agree(mid_model_path, monkeypatch):
    lens = [12, 47, 90]
    steps = 16
    rm = _load(mid_model_path, monkeypatch, persistent=False)
    assert rm.batch_decoder_kind == "rows"
    pm = _load(mid_model_path, monkeypatch, persistent=True)
    rc, _, _ = _prefilled(rm, None, lens, steps + 2)
    pc, _, _ = _prefilled(pm, None, lens, steps + 2)
    firsts = [int(x) for x in randmodel.prompt_ids(len(lens), rm.config.vocab_size, seed=77)]
    a = rm.decode_batch(firsts, lens, steps, rc)
    b = pm.decode_batch(firsts, lens, steps, pc)
    agree = (a == b).mean()
    assert agree >= 0.9, (a, b)  # low-margin steps may flip between the two summation orders


def test_persistent_batch_is_deterministic(mid_model_path, monkeypatch):
    gm = _load(mid_model_path, monkeypatch)
    lens = [10, 20, 30, 40, 50]
    runs = []
    for _ in range(2):
        gcs, _, _ = _prefilled(gm, None, lens, 12)
        runs.append(gm.decode_batch([1, 2, 3, 4, 5], lens, 10, gcs))
    assert (runs[0] == runs[1]).all()


def test_persistent_batch_bad_first_token(tiny_model_path, monkeypatch):
    gm = _load(tiny_model_path, monkeypatch)
    cs = [ci.CudaKVCache(gm, 16) for _ in range(2)]
    for c in cs:
        gm.prefill([1, 2, 3], 0, c, logits=False)
    # the host check refuses an id >= vocab before any launch
    with pytest.raises(ci.QwError) as e:
        gm.decode_batch([4, gm.config.vocab_size], [3, 3], 2, cs)
    assert e.value.code == ci.QW_ERR_ARG


def test_persistent_batch_expired_wait_is_reported_and_recovers(mid_model_path, monkeypatch):
    """The batch kernel's bounded waits, as for the decode kernels: with QW_TEST_STALL_CTA one CTA
    never raises its first end-of-step flag, every CTA's barrier wait expires (QW_WAIT_TIMEOUT_MS
    at its 50 ms floor), and the launch ends on its own with QW_ERR_DEVICE_TIMEOUT. The next
    batch decode on the same handle gives the same tokens as a model that never stalled."""
    monkeypatch.setenv("QW_BATCH_DECODER", "persistent")
    ref = ci.CudaModel.load_model(mid_model_path)
    monkeypatch.setenv("QW_TEST_STALL_CTA", "7")
    monkeypatch.setenv("QW_WAIT_TIMEOUT_MS", "50")
    gm = ci.CudaModel.load_model(mid_model_path)
    assert gm.batch_decoder_kind == "persistent"
    lens = [9, 17]
    gcs, _, _ = _prefilled(gm, None, lens, 12)
    with pytest.raises(ci.QwError) as e:
        gm.decode_batch([3, 4], lens, 4, gcs)
    assert e.value.code == ci.QW_ERR_DEVICE_TIMEOUT
    gcs, _, _ = _prefilled(gm, None, lens, 12)
    rcs, _, _ = _prefilled(ref, None, lens, 12)
    assert (gm.decode_batch([3, 4], lens, 6, gcs) == ref.decode_batch([3, 4], lens, 6, rcs)).all()
