"""The materialisation fused with the final layer's RMSNorm + modulate
(final_accumulate_reference, local_thc.py:1368-1372 / 1416-1420, then
FinalLayerSharedAdaLN.forward without its Linear, :865-873), inference only,
through the operator layer / C ABI.

The fused kernel rounds X_L to the activation dtype exactly as the
materialisation stores it and then follows the final-layer kernel's arithmetic
op by op; only the per-token sum of squares runs in another order (64-channel
slice sums added in slice order).  So it agrees with the two-kernel path (and
with the oracle's materialise + final_fwd) except for elements that a last-ulp
change of the fp32 norm moves across a rounding boundary of the dtype:
> 99.9 % identical in 16-bit, within the dtype tolerance everywhere.
"""
from __future__ import annotations

import pytest
import torch

from conftest import import_reference
from flowmatching_lthc_b200 import integration, ops
from oracle import lthc_oracle as O

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.bfloat16, torch.float16]
TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 2e-3}
# (B, G, C, L): the B/4 shape at small batch; one slice (cluster of 1) with a ragged
# channel slice; 4 slices; 16 slices (C = 1024) with ragged strips (G = 5); L = 1
SHAPES = [(2, 16, 768, 12), (1, 4, 40, 3), (3, 8, 256, 12), (1, 5, 1024, 12), (2, 16, 512, 1)]


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.detach().cpu().double(), b.detach().cpu().double()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def exact_fraction(a: torch.Tensor, b: torch.Tensor) -> float:
    return (a.detach().cpu() == b.detach().cpu()).float().mean().item()


def make(B, G, C, L, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x0 = torch.randn(B, 4 * G, 4 * G, C, generator=g).to(dtype)
    dz = [(0.1 * torch.randn(B, G * G, C, generator=g)).to(dtype) for _ in range(L)]
    betas = [0.02 * torch.randn(C, 16, generator=g) for _ in range(L)]  # fp32, as the released op takes them
    nw = 1.0 + 0.1 * torch.randn(C, generator=g)
    t2 = (0.5 * torch.randn(B, 2 * C, generator=g)).to(dtype)
    return x0, dz, betas, nw, t2


def two_kernel(x0, dz, betas, nw, shift, scale, eps=1e-6):
    xl = ops.materialise(x0, dz, betas)
    b, h, w, c = xl.shape
    return ops.final_norm_modulate(xl.reshape(b, h * w, c), nw, shift, scale, eps).reshape(b, h, w, c)


def check(ours, ref, dtype):
    assert ours.dtype == ref.dtype and ours.shape == ref.shape
    assert rel_err(ours, ref) < TOL[dtype]
    if dtype != torch.float32:
        assert exact_fraction(ours, ref) > 0.999


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("B, G, C, L", SHAPES)
def test_matches_two_kernel_path_and_oracle(B, G, C, L, dtype):
    x0, dz, betas, nw, t2 = make(B, G, C, L, dtype, seed=B * 100 + G * 10 + C + L)
    cu = [t.cuda() for t in (x0, nw, t2)]
    dzc, bc = [t.cuda() for t in dz], [t.cuda() for t in betas]
    shift, scale = cu[2].chunk(2, dim=1)  # strided rows, as the model passes them
    m = ops.materialise_final(cu[0], dzc, bc, cu[1], shift, scale, 1e-6)
    check(m, two_kernel(cu[0], dzc, bc, cu[1], shift, scale), dtype)
    xl = O.materialise(x0, dz, betas)
    ref = O.final_fwd(xl.reshape(B, 16 * G * G, C), nw, t2[:, :C], t2[:, C:], 1e-6).reshape(m.shape)
    check(m, ref, dtype)


def test_full_batch_b4_shape_and_determinism():
    x0, dz, betas, nw, t2 = make(64, 16, 768, 12, torch.bfloat16, seed=7)
    x0, nw, t2 = x0.cuda(), nw.cuda(), t2.cuda()
    dz, betas = [t.cuda() for t in dz], [t.cuda() for t in betas]
    shift, scale = t2.chunk(2, dim=1)
    m1 = ops.materialise_final(x0, dz, betas, nw, shift, scale, 1e-6)
    m2 = ops.materialise_final(x0, dz, betas, nw, shift, scale, 1e-6)
    assert torch.equal(m1, m2)
    check(m1, two_kernel(x0, dz, betas, nw, shift, scale), torch.bfloat16)
    assert ops.materialise_final_supported(x0, 12)


def test_validation():
    x0, dz, betas, nw, t2 = make(1, 4, 64, 2, torch.float32, seed=3)
    x0, nw, t2 = x0.cuda(), nw.cuda(), t2.cuda()
    dz, betas = [t.cuda() for t in dz], [t.cuda() for t in betas]
    shift, scale = t2.chunk(2, dim=1)
    with pytest.raises(ValueError):
        ops.materialise_final(x0, dz, betas, nw, shift.half(), scale, 1e-6)  # modulation dtype
    with pytest.raises(ValueError):
        ops.materialise_final(x0, dz, betas[:1], nw, shift, scale, 1e-6)     # one beta per layer
    with pytest.raises(ValueError):
        ops.materialise_final(x0, dz, betas, nw[:32], shift, scale, 1e-6)    # norm weight [C]
    big = torch.zeros(1, 16, 16, 1032, device="cuda")
    assert not ops.materialise_final_supported(big, 12)                       # C > 1024


def _small_model(L):
    from test_model_gpu import small_model
    return small_model(L)


@pytest.mark.parametrize("released", [False, True])
def test_model_inference_fused_equals_unfused(released, monkeypatch):
    """The installed inference forward with the fused final step against the same
    forward with the two calls (and, for the released B/4 model under bf16
    autocast, against the reference's own eager + Triton forward)."""
    L = import_reference()
    from test_model_gpu import inputs, reseed

    if released:
        from flowmatching_lthc.models import build_model
        torch.manual_seed(0)
        m = build_model("lthc_b4_velocity").cuda()
        reseed(m, 2)
        x, t, y = inputs(2, 256, seed=4)
        ctx, tol = torch.autocast("cuda", dtype=torch.bfloat16), 2e-2
    else:
        m = _small_model(L)
        x, t, y = inputs(2, 64, seed=4)
        ctx, tol = torch.autocast("cuda", enabled=False), 1e-5
    calls = []
    fused_op = ops.materialise_final
    monkeypatch.setattr(ops, "materialise_final", lambda *a: calls.append(1) or fused_op(*a))
    saved = integration.FUSE_FINAL
    with torch.no_grad(), ctx:
        ref = m(x, t, y)
        with integration.install(L):
            try:
                integration.FUSE_FINAL = True
                fused = m(x, t, y)
                integration.FUSE_FINAL = False
                unfused = m(x, t, y)
            finally:
                integration.FUSE_FINAL = saved
    assert len(calls) == 1  # the fused kernel ran for the FUSE_FINAL forward only
    assert ref.abs().max() > 0
    assert rel_err(fused, unfused) < tol
    assert rel_err(fused, ref) < tol


@pytest.mark.parametrize("dtype", DTYPES)
def test_empty_batch_and_smallest_channel_count(dtype):
    x0, dz, betas, nw, t2 = make(0, 4, 64, 2, dtype, seed=5)
    cu = lambda t: t.cuda()  # noqa: E731
    shift, scale = cu(t2).chunk(2, dim=1)
    m = ops.materialise_final(cu(x0), [cu(t) for t in dz], [cu(t) for t in betas], cu(nw), shift, scale, 1e-6)
    assert m.shape == x0.shape
    x0, dz, betas, nw, t2 = make(3, 4, 8, 2, dtype, seed=6)  # C = 8: one slice, 4 valid lanes
    t2c = cu(t2)
    m = ops.materialise_final(cu(x0), [cu(t) for t in dz], [cu(t) for t in betas], cu(nw), t2c[:, :8], t2c[:, 8:],
                              1e-6)
    check(m, two_kernel(cu(x0), [cu(t) for t in dz], [cu(t) for t in betas], cu(nw), t2c[:, :8], t2c[:, 8:]), dtype)
