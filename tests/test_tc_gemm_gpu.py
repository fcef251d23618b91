"""The prefill's tcgen05 tensor-core GEMM through the C ABI (qw_gemm_bf16x2), against a float64
product of the same bf16 operands: Y = (A_hi + A_lo) . B^T, with A_hi + A_lo the two-bf16 split of
f32 activations. Shapes cover the prefill's projections (K = 1024, 2048, 3072), a ragged M (rows
that are not a multiple of the 128-row tile, which the TMA zero-fills), the lm_head width and an
odd output width (rows of the f32 output that are not 16-byte aligned), and the few-row shapes of a
decode batch."""
from __future__ import annotations

import pytest

import cuda_inference as ci

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def split_bf16(a: "torch.Tensor"):
    hi = a.to(torch.bfloat16)
    lo = (a - hi.float()).to(torch.bfloat16)
    return hi.contiguous(), lo.contiguous()


# M <= 16 takes the swapped-operand (skinny) kernel: weights as the MMA's 128-row operand
@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (512, 4096, 1024), (200, 1024, 2048), (77, 6144, 1024),
                                   (512, 1024, 3072), (33, 151936, 1024), (130, 10007, 1024),
                                   (1, 4096, 1024), (8, 1024, 2048), (16, 6144, 1024), (5, 10007, 1024),
                                   (16, 1024, 3072), (3, 151936, 1024)])
def test_gemm_matches_f64(M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    a = torch.randn(M, K, device="cuda", generator=g)
    b = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    hi, lo = split_bf16(a)
    y = torch.full((M, N), float("nan"), device="cuda")
    ci.gemm_bf16x2(0, hi.data_ptr(), lo.data_ptr(), b.data_ptr(), y.data_ptr(), M, N, K)
    ref = (hi.double() + lo.double()) @ b.double().T
    err = (y.double() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 2e-5 * max(1.0, scale), (err, scale)
    # the split keeps ~16 bits of each activation: close to the f32 product too
    assert (y.double() - a.double() @ b.double().T).abs().max().item() <= 1e-3 * max(1.0, scale)


def test_gemm_rejects_bad_k():
    x = torch.zeros(128, 96, dtype=torch.bfloat16, device="cuda")
    y = torch.zeros(128, 128, device="cuda")
    with pytest.raises(ci.QwError) as e:
        ci.gemm_bf16x2(0, x.data_ptr(), x.data_ptr(), x.data_ptr(), y.data_ptr(), 128, 128, 96)
    assert e.value.code == ci.QW_ERR_ARG
