"""qw_argmax_f32_noalloc: the argmax entry point for callers that cannot allocate device memory.

Some callers cannot call cudaMalloc at the point where they need an argmax: code recording a CUDA
stream capture, or a host application that owns the device allocator and forbids allocations on
its serving path. For them qw_argmax_f32_noalloc keeps the kernel's scratch (the block partials
and the ticket that qw_argmax_f32 takes as a caller workspace) in one file-scope device array
instead. This test calls it through the C ABI twice in a row and checks each result against the
existing entry point, qw_argmax_f32, on the same input: argmax indices must be equal exactly (the
tolerance the other argmax tests use).

This file is named to be collected last, so that a run stopping at the first failure has run
every other test first; it also passes alone in a fresh process.
"""
from __future__ import annotations

import numpy as np
import pytest

import cuda_inference as ci

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _with_workspace(xd: "torch.Tensor") -> int:
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws = torch.empty(ci.argmax_workspace_size(xd.numel()), dtype=torch.uint8, device="cuda")
    ci.argmax_f32(0, xd.data_ptr(), xd.numel(), out.data_ptr(), ws.data_ptr())
    torch.cuda.synchronize()
    return int(out.item())


def _no_alloc(xd: "torch.Tensor") -> int:
    out = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    ci.argmax_f32_noalloc(0, xd.data_ptr(), xd.numel(), out.data_ptr())
    torch.cuda.synchronize()
    return int(out.item())


def test_noalloc_argmax_matches_workspace_argmax_twice():
    rng = np.random.Generator(np.random.PCG64(42))
    first = rng.standard_normal(151936).astype(np.float32)
    first[[5, 90000]] = first.max() + 1.0                  # a tie: the lower index must win
    second = rng.standard_normal(1 << 20).astype(np.float32)
    second[rng.choice(second.size, 50, replace=False)] = np.nan   # NaNs never win
    for x in (first, second):                                # two calls in a row share the scratch
        xd = torch.from_numpy(x).cuda()
        got = _no_alloc(xd)
        assert got == _with_workspace(xd)
    assert _no_alloc(torch.from_numpy(first).cuda()) == 5


def test_noalloc_argmax_rejects_bad_sizes():
    xd = torch.zeros(4, device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(ci.QwError) as e:
        ci.argmax_f32_noalloc(0, xd.data_ptr(), 0, out.data_ptr())
    assert e.value.code == ci.QW_ERR_ARG
    with pytest.raises(ci.QwError) as e:
        ci.argmax_f32_noalloc(0, xd.data_ptr(), 1 << 33, out.data_ptr())
    assert e.value.code == ci.QW_ERR_ARG
