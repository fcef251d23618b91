"""Batched prefill (qw_prefill, the 512-token prompt workload) against the reference CPU engine's token-by-token
prefill (the oracle, cpu_inference.rs:100-179): every position's logits within 1e-2 max-abs, the
K/V cache filled at the same slots (indexing exact, values within the f32 tolerance of the
reordered arithmetic), and a greedy decode continuing from a prefilled cache producing the same
tokens as one continuing from a forward-filled cache."""
from __future__ import annotations

import numpy as np
import pytest

import cpu_oracle as co
import cuda_inference as ci
import randmodel

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = 1e-2


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


# n = 300 and 600 reach query tiles whose positions span more than one attention split (192
# positions), so those cases also check the split merge
@pytest.mark.parametrize("geometry,n", [("tiny", 40), ("mid", 130), ("qwen3-0.6b", 64), ("mid", 300), ("tiny", 600)])
def test_prefill_matches_token_by_token_oracle(geometry, n):
    path = randmodel.make_model(geometry, 0)
    om = co.Model.load_model(path)
    oc = co.KVCache(om)
    ids = randmodel.prompt_ids(n, om.config.vocab_size, seed=3)
    want = np.stack([om.forward(t, p, oc) for p, t in enumerate(ids)])
    m = ci.CudaModel.load_model(path)
    cache = ci.CudaKVCache(m, n + 8)
    got = m.prefill(ids, 0, cache)
    assert got.shape == want.shape
    assert np.abs(got - want).max() <= TOL
    for l in (0, om.config.num_hidden_layers - 1):
        k, v = cache.layer(l, n)
        ko, vo = oc.layer(l)
        assert np.abs(k - ko).max() <= 1e-3 and np.abs(v - vo).max() <= 1e-3


def test_prefill_then_decode_matches_forward_then_decode(mid_model_path):
    m = ci.CudaModel.load_model(mid_model_path)
    ids = randmodel.prompt_ids(48, m.config.vocab_size, seed=5)
    c1, c2 = ci.CudaKVCache(m, 80), ci.CudaKVCache(m, 80)
    lg = m.prefill(ids, 0, c1)
    for p, t in enumerate(ids):
        lf = m.forward(t, p, c2)
    assert np.abs(lg[-1] - lf).max() <= TOL
    first = int(np.argmax(lf))
    assert m.decode(first, len(ids), 16, c1) == m.decode(first, len(ids), 16, c2)


def test_prefill_continues_an_existing_cache(mid_model_path):
    # two prefill calls (positions 0..19, then 20..49) equal one call over all 50 positions
    m = ci.CudaModel.load_model(mid_model_path)
    ids = randmodel.prompt_ids(50, m.config.vocab_size, seed=7)
    c1, c2 = ci.CudaKVCache(m, 64), ci.CudaKVCache(m, 64)
    whole = m.prefill(ids, 0, c1)
    m.prefill(ids[:20], 0, c2, logits=False)
    tail = m.prefill(ids[20:], 20, c2)
    assert np.abs(tail - whole[20:]).max() <= 1e-4


def test_prefill_continuation_across_attention_splits(mid_model_path):
    # the second call's tiles start at position 40 and read up to 330 positions, split differently
    # from the single call's: only the summation order of the softmax differs
    m = ci.CudaModel.load_model(mid_model_path)
    ids = randmodel.prompt_ids(330, m.config.vocab_size, seed=9)
    c1, c2 = ci.CudaKVCache(m, 336), ci.CudaKVCache(m, 336)
    whole = m.prefill(ids, 0, c1)
    m.prefill(ids[:40], 0, c2, logits=False)
    tail = m.prefill(ids[40:], 40, c2)
    assert np.abs(tail - whole[40:]).max() <= 1e-4


def test_prefill_argument_errors(tiny_model_path):
    m = ci.CudaModel.load_model(tiny_model_path)
    cache = ci.CudaKVCache(m, 16)
    with pytest.raises(ci.QwError) as e:
        m.prefill([1, 2, 3], 14, cache)                 # runs past the cache
    assert e.value.code == ci.QW_ERR_ARG
    with pytest.raises(ci.QwError) as e:
        m.prefill([1, m.config.vocab_size], 0, cache)   # token id out of range
    assert e.value.code == ci.QW_ERR_ARG
    # a device buffer as qw_prefill's host logits: refused before any work (qw_prefill_device takes those)
    ids = np.array([1, 2, 3], np.uint32)
    d_lg = torch.empty((3, m.config.vocab_size), dtype=torch.float32, device="cuda:0")
    assert ci.lib().qw_prefill(m._h, cache._h, ids.ctypes.data, 3, 0, d_lg.data_ptr()) == ci.QW_ERR_ARG


def test_prefill_device_bad_id_is_reported(tiny_model_path):
    """qw_prefill_device reads its ids from device memory, which the host cannot check: an id >=
    vocab_size is never used as an embedding row (row 0 is read instead) and the next qw_sync
    reports QW_ERR_ARG; the handle keeps working afterwards."""
    m = ci.CudaModel.load_model(tiny_model_path)
    cache = ci.CudaKVCache(m, 16)
    V = m.config.vocab_size
    d_ids = torch.tensor([3, V + 7, 5, -1], dtype=torch.int32, device="cuda")   # -1: 0xFFFFFFFF as uint32
    torch.cuda.synchronize()
    m.prefill_device(cache, d_ids.data_ptr(), 4, 0)
    with pytest.raises(ci.QwError) as e:
        m.sync()
    assert e.value.code == ci.QW_ERR_ARG
    m.sync()                                                 # the report was cleared
    ids = [3, 1, 5, 2]
    lg = m.prefill(ids, 0, ci.CudaKVCache(m, 16))
    assert np.isfinite(lg).all()


def test_prefill_logits_copy_paths_agree(full_model_path):
    """qw_prefill hands the logits to host memory in three ways: one DMA into a page-locked
    buffer, and, for pageable memory, two pinned stages that host threads copy out (into a new
    array, whose pages those threads touch first, or into an array written before). Each gives
    exactly the bytes that the device-side call leaves in device memory."""
    m = ci.CudaModel.load_model(full_model_path)
    V = m.config.vocab_size
    n = 200  # 121.5 MB of logits: seven full 16 MB stages and a partial one
    ids = randmodel.prompt_ids(n, V, seed=9)
    fresh = m.prefill(ids, 0, ci.CudaKVCache(m, n))
    reused = np.full((n, V), np.nan, np.float32)
    assert m.prefill(ids, 0, ci.CudaKVCache(m, n), out=reused) is reused
    pinned = torch.empty((n, V), dtype=torch.float32).pin_memory().numpy()
    pinned.fill(np.nan)
    assert m.prefill(ids, 0, ci.CudaKVCache(m, n), out=pinned) is pinned
    d_ids = torch.tensor(ids, dtype=torch.int32, device="cuda:0")
    d_lg = torch.empty((n, V), dtype=torch.float32, device="cuda:0")
    m.prefill_device(ci.CudaKVCache(m, n), d_ids.data_ptr(), n, 0, d_lg.data_ptr())
    m.sync()
    want = d_lg.cpu().numpy()
    for got in (fresh, reused, pinned):
        assert np.array_equal(got, want)
    with pytest.raises(ValueError):
        m.prefill(ids, 0, ci.CudaKVCache(m, n), out=np.empty((n, V), np.float64))
    with pytest.raises(ValueError):
        m.prefill(ids, 0, ci.CudaKVCache(m, n), out=np.empty((n - 1, V), np.float32))
