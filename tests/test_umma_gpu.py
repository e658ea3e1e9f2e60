"""The tensor-core (tcgen05 / TMEM) building blocks: a 128 x N x K bf16 GEMM on
one CTA through the operand descriptors the fused tensor-core kernels use,
against an fp32 torch matmul of the same bf16 operands (products are exact in
fp32; only the accumulation order differs)."""
from __future__ import annotations

import ctypes

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


# ---- no-swizzle operand layouts (the tensor-core materialisation backward) ----
# A core matrix is 8 rows x 16 bytes stored contiguously (128 bytes).  K-major:
# a row is one M (or N) index, its 16 bytes 8 consecutive K elements.  MN-major:
# a row is one K index, its 16 bytes 8 consecutive M (or N) elements.  In both,
# the descriptor's stride byte offset (SBO) steps between core matrices along
# M / N and its leading byte offset (LBO) along K.

def nosw_desc(start: int, lbo: int, sbo: int) -> int:
    return ((start >> 4) & 0x3FFF) | (((lbo >> 4) & 0x3FFF) << 16) | (((sbo >> 4) & 0x3FFF) << 32) | (1 << 46)


def idesc_f16(M: int, N: int, a_mn: bool, b_mn: bool, bf16: bool = True) -> int:
    fmt = 1 if bf16 else 0
    return (1 << 4) | (fmt << 7) | (fmt << 10) | (int(a_mn) << 15) | (int(b_mn) << 16) | ((N >> 3) << 17) | \
        ((M >> 4) << 24)


def nosw_image(mat: torch.Tensor, mn_major: bool, s_mn: int, s_k: int, nbytes: int) -> torch.Tensor:
    """Byte image of mat[MN, K] (16-bit) in the no-swizzle layout with core-matrix
    strides s_mn (along MN) and s_k (along K)."""
    MN, K = mat.shape
    img = torch.zeros(nbytes // 2, dtype=mat.dtype)
    mn = torch.arange(MN)[:, None].expand(MN, K)
    k = torch.arange(K)[None, :].expand(MN, K)
    inner = (k % 8) * 16 + (mn % 8) * 2 if mn_major else (mn % 8) * 16 + (k % 8) * 2
    off = (mn // 8) * s_mn + (k // 8) * s_k + inner
    img[(off // 2).reshape(-1)] = mat.reshape(-1)
    return img


def run_probe(A, B, a_mn, b_mn, a_str, b_str, steps, bf16=True, a_bytes=65536, b_bytes=65536):
    """D = A[128, K] @ B[N, K]^T through `steps` MMAs of K = 16 each."""
    N = B.shape[0]
    a_img = nosw_image(A, a_mn, *a_str, a_bytes).cuda()
    b_img = nosw_image(B, b_mn, *b_str, b_bytes).cuda()
    # a K step of 16 elements is two core matrices along K
    a_desc = (ctypes.c_uint64 * steps)(*[nosw_desc(2 * s * a_str[1], a_str[1], a_str[0]) for s in range(steps)])
    b_desc = (ctypes.c_uint64 * steps)(*[nosw_desc(2 * s * b_str[1], b_str[1], b_str[0]) for s in range(steps)])
    D = torch.full((128, N), float("nan"), device="cuda")
    status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    _lib.call("lthc_selftest_umma_desc", a_img.data_ptr(), a_bytes, b_img.data_ptr(), b_bytes, a_desc, b_desc, steps,
              idesc_f16(128, N, a_mn, b_mn, bf16), N, D.data_ptr(), status.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert status.item() == 0
    return D.cpu()


@pytest.mark.parametrize("bf16", [True, False])
@pytest.mark.parametrize("steps", [1, 2])
def test_no_swizzle_k_major_per_channel_gemm(bf16, steps):
    """Per-channel pooling GEMM: A = one channel's [128 cells x 16 positions]
    (cell groups 128 B apart, position halves 2 KB apart), B = [16 layers x 16
    positions] weights (layer groups 256 B apart, position halves 128 B apart)."""
    dt = torch.bfloat16 if bf16 else torch.float16
    g = torch.Generator().manual_seed(7 + steps)
    K = 16 * steps
    A = torch.randn(128, K, generator=g).to(dt)
    B = torch.randn(16, K, generator=g).to(dt)
    D = run_probe(A, B, False, False, (128, 2048), (256, 128 if steps == 1 else 512), steps, bf16)
    ref = A.float() @ B.float().T
    assert ((D - ref).abs().max() / ref.abs().max()).item() < 1e-5


def test_no_swizzle_mn_major_weight_gradient_gemm():
    """Weight-gradient GEMM: A[(channel, position) = 128, cells] MN-major (position
    halves 2 KB apart, cell groups 128 B apart), B[(layer, channel) = 96, cells]
    MN-major (layers 512 B apart, cell groups 128 B apart), K = 32 cells."""
    g = torch.Generator().manual_seed(11)
    A = torch.randn(128, 32, generator=g).to(torch.bfloat16)
    B = torch.randn(96, 32, generator=g).to(torch.bfloat16)
    D = run_probe(A, B, True, True, (2048, 128), (512, 128), 2)
    ref = A.float() @ B.float().T
    assert ((D - ref).abs().max() / ref.abs().max()).item() < 1e-5
