"""GPU test of lthc_weight_grad_noalloc, the weight-gradient entry point for
callers that cannot allocate device memory on the call path (hosts that give an
operator only its input and output buffers, or paths where a cudaMalloc would
synchronise the device).  It keeps its partial sums in a fixed buffer inside the
library instead of a caller workspace.

The test calls it through the C ABI twice in a row, on different inputs (so a
second call that reused stale contents of the shared buffer would be caught).
Both entry points run the same kernels in the same fixed reduction order and
differ only in where the partial sums live, so each result must equal
lthc_weight_grad's (given a normal workspace) bit for bit; it is also checked
against the CPU oracle's weight gradient at the tolerance the other
weight-gradient tests use (the oracle sums in another order).  A shape whose
partial sums do not fit the buffer must be refused before anything runs.
This file is collected last so that a failure here stops a -x run only after
every other test has run; it needs nothing from the other test files.
"""
from __future__ import annotations

import pytest
import torch

from flowmatching_lthc_b200 import _lib
from oracle import lthc_oracle as O

pytestmark = pytest.mark.gpu

RTOL_REDUCTION = 1e-5
BF16 = _lib.DTYPE_BF16


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def inputs(B: int, G: int, C: int, L: int, seed: int):
    g = torch.Generator(device="cuda").manual_seed(seed)
    high = torch.randn(B, 4 * G, 4 * G, C, device="cuda", generator=g).to(torch.bfloat16)
    low = [torch.randn(B, G * G, C, device="cuda", generator=g).to(torch.bfloat16) for _ in range(L)]
    return high, low


def with_workspace(high, low, B, G, C):
    L = len(low)
    lib = _lib.load()
    out = torch.empty(L, C, 16, device="cuda", dtype=torch.float32)
    nbytes = lib.lthc_weight_grad_workspace_bytes(B, G, C, L)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device="cuda")
    _lib.call("lthc_weight_grad", high.data_ptr(), _lib.ptr_array([t.data_ptr() for t in low]), L, out.data_ptr(),
              ws.data_ptr(), nbytes, B, G, C, BF16, torch.cuda.current_stream().cuda_stream)
    return out


def without_workspace(high, low, B, G, C):
    L = len(low)
    out = torch.full((L, C, 16), float("nan"), device="cuda", dtype=torch.float32)
    _lib.call("lthc_weight_grad_noalloc", high.data_ptr(), _lib.ptr_array([t.data_ptr() for t in low]), L,
              out.data_ptr(), B, G, C, BF16, torch.cuda.current_stream().cuda_stream)
    return out


@pytest.mark.parametrize("B,G,C,L", [(8, 16, 768, 1), (4, 16, 256, 3), (3, 5, 72, 2)])
def test_noalloc_weight_grad_matches_the_workspace_entry_point_on_two_calls(B, G, C, L):
    for call, seed in enumerate((11, 12)):
        high, low = inputs(B, G, C, L, seed + 100 * L)
        ref = with_workspace(high, low, B, G, C)
        got = without_workspace(high, low, B, G, C)
        torch.cuda.synchronize()
        assert torch.isfinite(got).all(), f"call {call}: output not fully written"
        assert torch.equal(got, ref), f"call {call}: differs from lthc_weight_grad"
        want = O.weight_grad(high.cpu(), [t.cpu() for t in low])
        assert rel_err(got, want) < RTOL_REDUCTION, f"call {call}: differs from the oracle"


def test_noalloc_refuses_shapes_beyond_its_buffer():
    B, G, C, L = 2, 16, 768, 12  # 12 layers of partials at C = 768 need far more than the fixed buffer
    high, low = inputs(B, G, C, L, 7)
    out = torch.full((L, C, 16), 3.0, device="cuda", dtype=torch.float32)
    with pytest.raises(_lib.LthcError) as ei:
        _lib.call("lthc_weight_grad_noalloc", high.data_ptr(), _lib.ptr_array([t.data_ptr() for t in low]), L,
                  out.data_ptr(), B, G, C, BF16, torch.cuda.current_stream().cuda_stream)
    assert ei.value.status == 5 and "fixed" in str(ei.value)
    torch.cuda.synchronize()
    assert bool((out == 3.0).all())  # nothing was enqueued
