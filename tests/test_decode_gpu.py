"""GPU parity: the B200 decode kernel against the CPU oracle, through the C ABI.

Ports the rules of the reference's tests/metal_parity.rs to seeded random-init weights:
  * metal_matches_cpu (:16-40): per position, logits finite and max |cpu - gpu| < 1e-2, and the
    same greedy token (here: unless the oracle's top-2 margin is below 1e-2, where a float
    reordering may legitimately flip it);
  * pipelined_decode_matches_forward (:44-71): decode()'s on-GPU argmax chain equals forward()
    plus the CPU argmax, exactly, over 48 steps.
Plus KV-cache indexing against the oracle's cache, determinism, argument errors, and the
long-context split-K path (config 2's 2048-token prompt on the per-layer Qwen3-0.6B shapes).
"""
from __future__ import annotations

import numpy as np
import pytest

import cpu_oracle as co
import cuda_inference as ci
import randmodel

pytestmark = pytest.mark.gpu

MAX_ABS_DIFF = 1e-2   # metal_parity.rs:14
MARGIN = 1e-2         # greedy tokens must agree where the oracle's top-2 gap is at least this


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _parity(path, n_tokens, seed=1, max_seq=None):
    cpu = co.Model.load_model(path)
    gpu = ci.CudaModel.load_model(path)
    cc = co.KVCache(cpu)
    gc = ci.CudaKVCache(gpu, max_seq or n_tokens + 1)
    ids = randmodel.prompt_ids(n_tokens, cpu.config.vocab_size, seed)
    worst = 0.0
    for pos, tok in enumerate(ids):
        a = cpu.forward(tok, pos, cc)
        b = gpu.forward(tok, pos, gc)
        assert a.shape == b.shape
        assert np.isfinite(b).all(), f"non-finite logits at pos {pos}"
        diff = float(np.abs(a - b).max())
        worst = max(worst, diff)
        assert diff < MAX_ABS_DIFF, f"pos {pos}: logits diverge by {diff}"
        if co.top2_margin(a) >= MARGIN:
            assert co.argmax(a) == co.argmax(b), f"pos {pos}: different greedy token"
    return cpu, gpu, cc, gc, ids, worst


@pytest.mark.parametrize("geometry,n", [("tiny", 24), ("mid", 24), ("qwen3-0.6b", 10)])
def test_cuda_matches_cpu(geometry, n):
    path = randmodel.make_model(geometry, 0)
    *_, worst = _parity(path, n)
    print(f"{geometry}: max |cpu - gpu| = {worst:.3e}")


@pytest.mark.parametrize("ctas", [100, 37])
def test_uneven_row_partition(ctas, monkeypatch):
    """Fewer CTAs than SMs (QW_CTAS, read at load): the 64-byte output units then fall unevenly
    (100 CTAs: 8 or 16 x rows each; 37 CTAs: phase rows spanning more ring pieces than the ring
    holds), and forward() and decode() must still match the oracle."""
    monkeypatch.setenv("QW_CTAS", str(ctas))
    cpu, gpu, cc, gc, ids, worst = _parity(randmodel.make_model("mid", 0), 12, max_seq=24)
    assert gpu.num_ctas == ctas
    logits = gpu.forward(ids[-1], len(ids), gc)
    expected = cpu.forward(ids[-1], len(ids), cc)
    assert float(np.abs(expected - logits).max()) < MAX_ABS_DIFF
    tok = co.argmax(logits)
    got = gpu.decode(tok, len(ids) + 1, 4, gc)
    for i, t in enumerate(got):
        ref = cpu.forward(tok, len(ids) + 1 + i, cc)
        if co.top2_margin(ref) < MARGIN:
            break
        assert t == co.argmax(ref), f"step {i}"
        tok = t
    print(f"{ctas} CTAs: max |cpu - gpu| = {worst:.3e}")


def test_kv_cache_matches_oracle(mid_model_path):
    cpu, gpu, cc, gc, ids, _ = _parity(mid_model_path, 12, seed=3, max_seq=20)
    n = len(ids)
    for layer in range(cpu.config.num_hidden_layers):
        ko, vo = cc.layer(layer)
        kg, vg = gc.layer(layer, n + 4)
        assert np.abs(kg[:n] - ko).max() < 1e-3
        assert np.abs(vg[:n] - vo).max() < 1e-3
        # nothing was written past the last position (KV indexing)
        assert not kg[n:].any() and not vg[n:].any()


def test_pipelined_decode_matches_forward(full_model_path):
    # metal_parity.rs:44-71, with enough context that attention has more positions than splits
    steps = 48
    gpu = ci.CudaModel.load_model(full_model_path)
    prompt = randmodel.prompt_ids(5, gpu.config.vocab_size, seed=11)
    max_seq = len(prompt) + steps + 1
    cache = ci.CudaKVCache(gpu, max_seq)
    logits = None
    for pos, tok in enumerate(prompt):
        logits = gpu.forward(tok, pos, cache)
    first = co.argmax(logits)
    expected, tok = [], first
    for i in range(steps):
        tok = co.argmax(gpu.forward(tok, len(prompt) + i, cache))
        expected.append(tok)
    cache = ci.CudaKVCache(gpu, max_seq)
    for pos, t in enumerate(prompt):
        gpu.forward(t, pos, cache)
    got = []
    gpu.decode(first, len(prompt), steps, cache, got.append)
    assert got == expected


def test_decode_is_deterministic(mid_model_path):
    gpu = ci.CudaModel.load_model(mid_model_path)
    ids = randmodel.prompt_ids(40, gpu.config.vocab_size, seed=5)
    runs = []
    for _ in range(2):
        cache = ci.CudaKVCache(gpu, 128)
        lg = [gpu.forward(t, p, cache) for p, t in enumerate(ids)]
        toks = gpu.decode(co.argmax(lg[-1]), len(ids), 60, cache)
        runs.append((np.stack(lg), toks))
    assert np.array_equal(runs[0][0], runs[1][0])  # bit-identical logits
    assert runs[0][1] == runs[1][1]


def test_traced_and_untraced_kernel_instances_agree(mid_model_path):
    """Tracing launches the kernel instance with the timeline stamps compiled in; the stamps are its
    only difference, so its logits and tokens are bit-identical to the untraced instance's."""
    gpu = ci.CudaModel.load_model(mid_model_path)
    ids = randmodel.prompt_ids(24, gpu.config.vocab_size, seed=9)
    runs = []
    for traced in (False, True):
        gpu.set_trace(traced)
        cache = ci.CudaKVCache(gpu, 64)
        lg = [gpu.forward(t, p, cache) for p, t in enumerate(ids)]
        toks = gpu.decode(co.argmax(lg[-1]), len(ids), 12, cache)
        runs.append((np.stack(lg), toks))
    gpu.set_trace(False)
    assert np.array_equal(runs[0][0], runs[1][0])
    assert runs[0][1] == runs[1][1]


def test_long_context_split_attention(mid_model_path):
    # config 2's shape of work: a 2048-token prompt fed token by token, then decode; the
    # attention splits each KV head's 2048+ positions over 18 CTAs and several ring slots each
    n_prompt, n_dec = 2048, 32
    cpu = co.Model.load_model(mid_model_path)
    gpu = ci.CudaModel.load_model(mid_model_path)
    cc, gc = co.KVCache(cpu), ci.CudaKVCache(gpu, n_prompt + n_dec + 1)
    ids = randmodel.prompt_ids(n_prompt, cpu.config.vocab_size, seed=2)
    check = set(range(0, n_prompt, 97)) | {n_prompt - 1}
    a = b = None
    for pos, tok in enumerate(ids):
        a = cpu.forward(tok, pos, cc)
        b = gpu.forward(tok, pos, gc)
        if pos in check:
            assert np.abs(a - b).max() < MAX_ABS_DIFF, pos
    # teacher-forced decode: both engines are fed the oracle's greedy token
    tok = co.argmax(a)
    for i in range(n_dec):
        pos = n_prompt + i
        a = cpu.forward(tok, pos, cc)
        b = gpu.forward(tok, pos, gc)
        assert np.abs(a - b).max() < MAX_ABS_DIFF, pos
        if co.top2_margin(a) >= MARGIN:
            assert co.argmax(a) == co.argmax(b)
        tok = co.argmax(a)


def test_argument_errors(tiny_model_path):
    gpu = ci.CudaModel.load_model(tiny_model_path)
    cache = ci.CudaKVCache(gpu, 8)
    with pytest.raises(ci.QwError) as e:
        gpu.forward(gpu.config.vocab_size, 0, cache)          # token out of range
    assert e.value.code == ci.QW_ERR_ARG
    with pytest.raises(ci.QwError) as e:
        gpu.forward(1, 8, cache)                              # metal_inference.rs:321 pos >= max_seq
    assert e.value.code == ci.QW_ERR_ARG
    with pytest.raises(ci.QwError) as e:
        gpu.decode(1, 4, 5, cache)                            # runs past the cache
    assert e.value.code == ci.QW_ERR_ARG
    other = ci.CudaModel.load_model(tiny_model_path)
    with pytest.raises(ci.QwError):
        other.forward(1, 0, cache)                            # cache of another model
    # the handle still works after the rejected calls
    assert np.isfinite(gpu.forward(1, 0, cache)).all()


def test_device_token_out_of_range_is_reported(tiny_model_path):
    import torch
    gpu = ci.CudaModel.load_model(tiny_model_path)
    cache = ci.CudaKVCache(gpu, 8)
    toks = torch.tensor([gpu.config.vocab_size + 5, 0, 0], dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    gpu.decode_device(cache, toks.data_ptr(), 0, 2)
    with pytest.raises(ci.QwError) as e:
        gpu.sync()
    assert e.value.code == ci.QW_ERR_ARG
    assert np.isfinite(gpu.forward(1, 0, cache)).all()     # recovered


def test_decoder_selection(full_model_path, mid_model_path, tiny_model_path, monkeypatch):
    """The grid kernel (one CTA per SM) is the default for every shape; QW_DECODER=cluster selects
    the cluster kernel (8 clusters x 8 CTAs) for the Qwen3-0.6B layer shape and is refused for others."""
    for path in (full_model_path, mid_model_path, tiny_model_path):
        m = ci.CudaModel.load_model(path)
        assert m.decoder_kind == "grid"
        m.close()
    monkeypatch.setenv("QW_DECODER", "cluster")
    for path in (full_model_path, mid_model_path):
        m = ci.CudaModel.load_model(path)
        assert m.decoder_kind == "cluster" and m.num_ctas == 64
        m.close()
    with pytest.raises(ci.QwError) as e:
        ci.CudaModel.load_model(tiny_model_path)
    assert e.value.code == ci.QW_ERR_UNSUPPORTED


def test_cluster_and_grid_kernels_agree(mid_model_path, monkeypatch):
    """The two decode kernels compute the same function with different summation orders: their
    logits agree far inside the oracle bar, and their greedy decodes give the same tokens."""
    gr = ci.CudaModel.load_model(mid_model_path)
    monkeypatch.setenv("QW_DECODER", "cluster")
    cl = ci.CudaModel.load_model(mid_model_path)
    assert (cl.decoder_kind, gr.decoder_kind) == ("cluster", "grid")
    ids = randmodel.prompt_ids(40, cl.config.vocab_size, seed=21)
    c1, c2 = ci.CudaKVCache(cl, 80), ci.CudaKVCache(gr, 80)
    worst = 0.0
    for pos, tok in enumerate(ids):
        a, b = cl.forward(tok, pos, c1), gr.forward(tok, pos, c2)
        worst = max(worst, float(np.abs(a - b).max()))
    assert worst < 1e-3, worst
    first = co.argmax(a)
    assert cl.decode(first, len(ids), 24, c1) == gr.decode(first, len(ids), 24, c2)
    print(f"cluster vs grid: max |diff| = {worst:.2e}")


def test_cluster_kernel_device_token_out_of_range(mid_model_path, monkeypatch):
    monkeypatch.setenv("QW_DECODER", "cluster")
    gpu = ci.CudaModel.load_model(mid_model_path)
    assert gpu.decoder_kind == "cluster"
    import torch
    cache = ci.CudaKVCache(gpu, 8)
    toks = torch.tensor([gpu.config.vocab_size + 5, 0, 0], dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    gpu.decode_device(cache, toks.data_ptr(), 0, 2)
    with pytest.raises(ci.QwError) as e:
        gpu.sync()
    assert e.value.code == ci.QW_ERR_ARG
    assert np.isfinite(gpu.forward(1, 0, cache)).all()     # recovered


@pytest.mark.parametrize("geometry,kind", [("mid", "cluster"), ("tiny", "grid")])
def test_expired_wait_is_reported_and_the_handle_recovers(geometry, kind, monkeypatch):
    """A bounded device wait that runs out: with the test hook QW_TEST_STALL_CTA one CTA never raises
    its first end-of-token flag, so every CTA's barrier wait expires (QW_WAIT_TIMEOUT_MS at its 50 ms
    floor). The launch must end on its own and report QW_ERR_DEVICE_TIMEOUT; the next calls on the
    same handle must give the same logits as a model that never stalled."""
    path = randmodel.make_model(geometry, 0)
    if kind == "cluster":
        monkeypatch.setenv("QW_DECODER", "cluster")
    ref = ci.CudaModel.load_model(path)
    monkeypatch.setenv("QW_TEST_STALL_CTA", "5")
    monkeypatch.setenv("QW_WAIT_TIMEOUT_MS", "50")
    gpu = ci.CudaModel.load_model(path)
    assert gpu.decoder_kind == kind
    cache = ci.CudaKVCache(gpu, 16)
    with pytest.raises(ci.QwError) as e:
        gpu.forward(3, 0, cache)
    assert e.value.code == ci.QW_ERR_DEVICE_TIMEOUT
    rc = ci.CudaKVCache(ref, 16)
    for pos, tok in enumerate([3, 7, 11]):
        a, b = gpu.forward(tok, pos, cache), ref.forward(tok, pos, rc)
        assert np.array_equal(a, b), pos
    assert gpu.decode(5, 3, 4, cache) == ref.decode(5, 3, 4, rc)
