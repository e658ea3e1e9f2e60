"""The tensor-core (tcgen05 / TMEM) building blocks: a 128 x N x K bf16 GEMM on
one CTA through the operand descriptors the fused tensor-core kernels use,
against an fp32 torch matmul of the same bf16 operands (products are exact in
fp32; only the accumulation order differs)."""
from __future__ import annotations

import pytest
import torch

from flowmatching_lthc_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("N", [64, 128, 256])
@pytest.mark.parametrize("K", [64, 128, 256])
def test_umma_selftest_gemm(N, K):
    g = torch.Generator().manual_seed(N * 1000 + K)
    A = torch.randn(128, K, generator=g).to(torch.bfloat16).cuda()
    B = torch.randn(N, K, generator=g).to(torch.bfloat16).cuda()
    D = torch.full((128, N), float("nan"), device="cuda")
    status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    _lib.call("lthc_selftest_umma", A.data_ptr(), B.data_ptr(), D.data_ptr(), N, K, status.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert status.item() == 0
    ref = A.float() @ B.float().T
    err = ((D - ref).abs().max() / ref.abs().max()).item()
    assert err < 1e-5, err


def test_umma_selftest_rejects_bad_shapes():
    with pytest.raises(_lib.LthcError):
        _lib.call("lthc_selftest_umma", 256, 256, 256, 96, 64, 256, None)
    with pytest.raises(_lib.LthcError):
        _lib.call("lthc_selftest_umma", 256, 256, 256, 128, 80, 256, None)
