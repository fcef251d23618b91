"""Standalone kernels through the C ABI: the decode kernel's GEMV machinery at benchmark config 3's
shapes against float64 accumulation, the argmax rule bit-exact against the oracle's
(tests/common/mod.rs:17-22), and the streaming-read probe (tests/read_bandwidth.rs:122-124)."""
from __future__ import annotations

import numpy as np
import pytest

import cpu_oracle as co
import cuda_inference as ci

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

GEMV_SHAPES = [(2048, 1024), (1024, 1024), (1024, 2048), (6144, 1024), (1024, 3072), (151936, 1024), (1000, 256), (37, 768)]


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.mark.parametrize("rows,cols", GEMV_SHAPES)
def test_gemv_matches_f64(rows, cols):
    g = torch.Generator().manual_seed(rows * 7 + cols)
    w = (torch.randn(rows, cols, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(cols, generator=g)
    ref = w.double() @ x.double()
    wd, xd = w.cuda(), x.cuda()
    yd = torch.full((rows,), float("nan"), device="cuda")
    ci.gemv_bf16(0, wd.data_ptr(), xd.data_ptr(), yd.data_ptr(), rows, cols)
    torch.cuda.synchronize()
    err = (yd.cpu().double() - ref).abs().max().item()
    # f32 accumulation of cols products of size ~0.02: error well below 1e-4
    assert err < 1e-4, err


@pytest.mark.parametrize("rows,cols,count", [(2048, 1024, 9), (1024, 2048, 5), (1024, 3072, 3), (37, 768, 4)])
def test_gemv_seq_matches_single_launches(rows, cols, count):
    """qw_gemv_bf16_seq (count stacked matrices in one launch) gives, bit for bit, what one
    qw_gemv_bf16 launch per matrix gives (same rows per CTA, same reduction order), and matches f64."""
    g = torch.Generator().manual_seed(rows + 13 * cols + count)
    w = (torch.randn(count, rows, cols, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(cols, generator=g)
    wd, xd = w.cuda(), x.cuda()
    ys = torch.full((count, rows), float("nan"), device="cuda")
    ci.gemv_bf16_seq(0, wd.data_ptr(), xd.data_ptr(), ys.data_ptr(), rows, cols, count)
    y1 = torch.full((count, rows), float("nan"), device="cuda")
    for m in range(count):
        ci.gemv_bf16(0, wd[m].data_ptr(), xd.data_ptr(), y1[m].data_ptr(), rows, cols)
    torch.cuda.synchronize()
    assert torch.equal(ys, y1)
    ref = torch.einsum("mrc,c->mr", w.double(), x.double())
    assert (ys.cpu().double() - ref).abs().max().item() < 1e-4


def _gpu_argmax(x: np.ndarray) -> int:
    xd = torch.from_numpy(x).cuda()
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws = torch.empty(ci.argmax_workspace_size(x.size), dtype=torch.uint8, device="cuda")
    ci.argmax_f32(0, xd.data_ptr(), x.size, out.data_ptr(), ws.data_ptr())
    torch.cuda.synchronize()
    return int(out.item())


def test_argmax_rule_bit_exact():
    rng = np.random.Generator(np.random.PCG64(0))
    cases = [
        np.array([1, 3, 3, 2], np.float32),
        np.array([np.nan, 5, 7], np.float32),
        np.array([1, np.nan, 7, np.nan], np.float32),
        np.array([-np.inf, -np.inf, -np.inf], np.float32),
        np.array([-np.inf, np.nan, -np.inf], np.float32),
        np.zeros(151936, np.float32),
        np.array([0.0], np.float32),
    ]
    for n in (151936, 10007, 1 << 20):
        x = rng.standard_normal(n).astype(np.float32)
        m = x.max()
        for idx in rng.choice(n, 3, replace=False):
            x[idx] = m + 1.0        # planted ties of the maximum at random positions
        cases.append(x)
        y = x.copy()
        y[rng.choice(n, 100, replace=False)] = np.nan
        cases.append(y)
    for x in cases:
        assert _gpu_argmax(x) == co.argmax(x), x[:8]


def test_read_probe_reads_every_element():
    n = 64 << 20
    src = torch.ones(n, device="cuda")
    parts = torch.zeros(4096, device="cuda")
    k = ci.read_probe(0, src.data_ptr(), n, parts.data_ptr(), parts.numel())
    torch.cuda.synchronize()
    assert parts[:k].double().sum().item() == float(n)
