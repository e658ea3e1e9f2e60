"""Fused final-layer prologue (RMSNorm + AdaLN modulate of FinalLayerSharedAdaLN,
local_thc.py:865-873) on the GPU, through the operator layer / C ABI.

The kernel follows the reference's rounding op by op; only the two sums over
channels (mean of squares, the backward's dot product) run in another order
than torch's.  So 16-bit outputs agree with the oracle and with the reference's
own eager code on the GPU exactly except for elements that a last-ulp change of
the fp32 norm moves across a bf16/fp16 rounding boundary (measured: > 99.9 %
exact; asserted: 99.9 % forward, 99 % grad x), and never by more than the
dtype tolerance (2e-2 bf16 of the largest magnitude).  fp32 outputs: 1e-5.
Sums over tokens (grad weight / shift / scale): 1e-5 relative in fp32 (grad
scale in 16-bit: 1e-3, its terms hold the rounded n).
"""
from __future__ import annotations

import pytest
import torch

from conftest import GOLDEN, import_reference
from flowmatching_lthc_b200 import ops
from oracle import lthc_oracle as O

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.bfloat16, torch.float16]
TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 2e-3}
RTOL_REDUCTION = 1e-5
# (B, T, C): the B/4 final layer (4096 tokens, 768 channels) at small batch, fewer
# tokens than warps in a CTA, a ragged last 256-channel chunk, minimum C, maximum C
SHAPES = [(2, 4096, 768), (3, 5, 768), (2, 64, 264), (4, 33, 8), (1, 128, 1024), (2, 96, 512)]


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.detach().cpu().double(), b.detach().cpu().double()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def exact_fraction(a: torch.Tensor, b: torch.Tensor) -> float:
    return (a.detach().cpu() == b.detach().cpu()).float().mean().item()


def inputs(B, T, C, dt, seed, chunked=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, C, generator=g).to(dt)
    w = torch.randn(C, generator=g) * 0.1 + 1.0
    t2 = (torch.randn(B, 2 * C, generator=g) * 0.5).to(dt)
    gm = torch.randn(B, T, C, generator=g).to(dt)
    x, w, t2, gm = x.cuda(), w.cuda(), t2.cuda(), gm.cuda()
    shift, scale = t2.chunk(2, dim=1)  # strided views, as FinalLayerSharedAdaLN passes them
    if not chunked:
        shift, scale = shift.contiguous(), scale.contiguous()
    return x, w, shift, scale, gm


def check_close(out, ref, dt, exact=0.999):
    assert out.dtype == ref.dtype and out.shape == ref.shape
    if dt != torch.float32:
        assert exact_fraction(out, ref) > exact
    assert rel_err(out, ref) < TOL[dt]


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("shape", SHAPES)
def test_forward_matches_oracle(shape, dt):
    B, T, C = shape
    x, w, shift, scale, _ = inputs(B, T, C, dt, seed=B * 7 + C)
    m = ops.final_norm_modulate(x, w, shift, scale, 1e-6)
    ref = O.final_fwd(x.cpu(), w.cpu(), shift.cpu(), scale.cpu(), 1e-6)
    check_close(m, ref, dt)


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("shape", SHAPES)
def test_backward_matches_oracle(shape, dt):
    B, T, C = shape
    x, w, shift, scale, gm = inputs(B, T, C, dt, seed=B * 11 + C, chunked=False)
    gx, gw, gsh, gsc = ops.final_norm_modulate_bwd(gm, x, w, scale, 1e-6)
    rx, rw, rsh, rsc = O.final_bwd(gm.cpu(), x.cpu(), w.cpu(), scale.cpu(), 1e-6)
    check_close(gx, rx, dt, exact=0.99)
    assert rel_err(gw, rw) < RTOL_REDUCTION
    assert rel_err(gsh, rsh) < RTOL_REDUCTION
    # grad scale sums round(g_m * n): an n that moved by one 16-bit ulp (above)
    # moves its term by one ulp, so 16-bit sums carry that much more spread
    assert rel_err(gsc, rsc) < (RTOL_REDUCTION if dt == torch.float32 else 1e-3)


def test_goldens_through_cuda():
    for name in ("final_t64_c768_bf16", "final_t16_c40_f32", "final_t8_c1024_bf16"):
        c = torch.load(GOLDEN / f"{name}.pt")
        C, eps, dt = c["meta"]["C"], c["meta"]["eps"], c["x"].dtype
        x, t2, w, gm = c["x"].cuda(), c["t2"].cuda(), c["norm_weight"].cuda(), c["g_m"].cuda()
        shift, scale = t2.chunk(2, dim=1)
        check_close(ops.final_norm_modulate(x, w, shift, scale, eps), c["m"], dt)
        gx, gw, gsh, gsc = ops.final_norm_modulate_bwd(gm, x, w, scale, eps)
        check_close(gx, c["gx"], dt, exact=0.99)
        assert rel_err(gw, c["g_norm_weight"]) < RTOL_REDUCTION
        assert rel_err(gsh.to(dt), c["g_shift"]) < TOL[dt]
        assert rel_err(gsc.to(dt), c["g_scale"]) < TOL[dt]


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_autograd_matches_reference_eager_on_gpu(dt):
    """The reference's own RMSNorm module and modulate, on the same GPU, at the B/4
    final-layer shape: forward and every gradient."""
    L = import_reference()
    B, T, C = 2, 4096, 768
    x, w, shift, scale, gm = inputs(B, T, C, dt, seed=99)
    norm = L.RMSNorm(C).cuda()
    with torch.no_grad():
        norm.weight.copy_(w)
    t2 = torch.cat([shift, scale], dim=1)

    xr, t2r = x.clone().requires_grad_(True), t2.clone().requires_grad_(True)
    sh, sc = t2r.chunk(2, dim=1)
    ref = L.modulate(norm(xr), sh, sc)
    ref.backward(gm)

    xo, wo, t2o = x.clone().requires_grad_(True), w.clone().requires_grad_(True), t2.clone().requires_grad_(True)
    sh, sc = t2o.chunk(2, dim=1)
    out = ops.final_norm_modulate(xo, wo, sh, sc, norm.eps)
    out.backward(gm)

    check_close(out, ref, dt)
    check_close(xo.grad, xr.grad, dt, exact=0.99)
    assert rel_err(wo.grad, norm.weight.grad) < RTOL_REDUCTION * 10
    assert rel_err(t2o.grad.float(), t2r.grad.float()) < TOL[dt]


def test_backward_is_deterministic():
    x, w, shift, scale, gm = inputs(4, 1000, 768, torch.bfloat16, seed=5)
    a = ops.final_norm_modulate_bwd(gm, x, w, scale, 1e-6)
    b = ops.final_norm_modulate_bwd(gm, x, w, scale, 1e-6)
    for u, v in zip(a, b):
        assert torch.equal(u, v)


def test_empty_and_validation():
    x, w, shift, scale, gm = inputs(2, 0, 768, torch.bfloat16, seed=1)
    assert ops.final_norm_modulate(x, w, shift, scale, 1e-6).shape == (2, 0, 768)
    gx, gw, gsh, gsc = ops.final_norm_modulate_bwd(gm, x, w, scale, 1e-6)
    assert gx.shape == (2, 0, 768) and not gw.any() and not gsh.any() and not gsc.any()
    x, w, shift, scale, gm = inputs(0, 16, 768, torch.bfloat16, seed=1)  # empty batch: [0, C] modulation rows
    assert ops.final_norm_modulate(x, w, shift, scale, 1e-6).shape == (0, 16, 768)
    gx, gw, gsh, gsc = ops.final_norm_modulate_bwd(gm, x, w, scale, 1e-6)
    assert gx.shape == (0, 16, 768) and gsh.shape == (0, 768) and not gw.any()
    x, w, shift, scale, _ = inputs(2, 8, 768, torch.bfloat16, seed=1)
    with pytest.raises(ValueError):
        ops.final_norm_modulate(x, w, shift.float(), scale.float(), 1e-6)  # dtype mix
    with pytest.raises((ValueError, NotImplementedError)):  # no CPU path (the op has only a CUDA kernel)
        ops.final_norm_modulate(x.cpu(), w.cpu(), shift.cpu(), scale.cpu(), 1e-6)
    x2, w2, s2, c2, _ = inputs(1, 4, 1032, torch.bfloat16, seed=2)
    with pytest.raises(ValueError):
        ops.final_norm_modulate(x2, w2, s2, c2, 1e-6)  # above the 1024-channel limit


def test_final_layer_patch_matches_reference_layer():
    """integration.install() routes FinalLayerSharedAdaLN.forward (norm + modulate
    fused, the Linear unchanged) and uninstall() restores it."""
    L = import_reference()
    from flowmatching_lthc_b200 import integration

    torch.manual_seed(0)
    layer = L.FinalLayerSharedAdaLN(768, 4, 3).cuda()
    with torch.no_grad():
        layer.linear.weight.normal_(0, 0.02)
        layer.norm_final.weight.normal_(1.0, 0.1)
    x, _, shift, scale, _ = inputs(2, 4096, 768, torch.bfloat16, seed=3)
    t2 = torch.cat([shift, scale], dim=1)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        ref = layer(x, t2)
        with integration.install(L):
            assert L.FinalLayerSharedAdaLN.forward is integration._final_layer
            out = layer(x, t2)
        assert L.FinalLayerSharedAdaLN.forward is not integration._final_layer
    assert rel_err(out, ref) < TOL[torch.bfloat16]
    assert exact_fraction(out, ref) > 0.9  # a flipped m element can move its token's Linear outputs by an ulp


def test_compiles_fullgraph():
    torch._dynamo.reset()
    x, w, shift, scale, gm = inputs(2, 64, 768, torch.bfloat16, seed=4)
    t2 = torch.cat([shift, scale], dim=1)

    def f(x, w, t2):
        sh, sc = t2.chunk(2, dim=1)
        return ops.final_norm_modulate(x, w, sh, sc, 1e-6)

    def run(fn):
        xa, wa, ta = x.clone().requires_grad_(True), w.clone().requires_grad_(True), t2.clone().requires_grad_(True)
        out = fn(xa, wa, ta)
        out.backward(gm)
        return [out, xa.grad, wa.grad, ta.grad]

    for e, c in zip(run(f), run(torch.compile(f, fullgraph=True))):
        assert torch.equal(e, c) or rel_err(c, e) < RTOL_REDUCTION
