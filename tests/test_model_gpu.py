"""Drop-in parity on the reference model: the released LTHC-B/4 model
(``build_model('lthc_b4_velocity')``) and a small shared-read model, run once
with the reference's own code and once with ``integration.install()`` routing
the LTHC interface through the B200 kernels.

The zero-initialised layers of the reference (AdaLN modulation, final linear)
make a freshly built model output exactly zero, so every test re-seeds them.
The reference's fused Triton op is hard-wired to the 64x64 residual grid, so it
only runs on B/4 shapes; the small model uses the reference's pure-PyTorch
accumulate loop.
"""
from __future__ import annotations

import pytest
import torch

from conftest import import_reference
from flowmatching_lthc_b200 import integration, workloads

pytestmark = pytest.mark.gpu


def rel_err(a, b) -> float:
    a, b = a.detach().float().cpu().double(), b.detach().float().cpu().double()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def reseed(model: torch.nn.Module, seed: int) -> None:
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("read_logits"):
                p.copy_(torch.randn(p.shape, generator=g))
            elif name.endswith("write_weight"):
                p.copy_(1.0 + 0.1 * torch.randn(p.shape, generator=g))
            elif torch.count_nonzero(p) == 0:
                p.copy_(0.02 * torch.randn(p.shape, generator=g))


def inputs(B: int, size: int, seed: int = 0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(B, 3, size, size, device="cuda", generator=g)
    t = torch.rand(B, device="cuda", generator=g)
    y = torch.randint(0, 1000, (B,), device="cuda", generator=g)
    return x, t, y


def small_model(L):
    torch.manual_seed(0)
    m = L.SharedReadLocalTHCSharedAdaLNJiT(input_size=64, patch_size=4, hidden_size=64, depth=12, num_heads=4,
                                            workspace_grid=4, bottleneck_dim=32, attn_backend="math").cuda()
    reseed(m, 1)
    return m


def test_small_model_forward_fp32_lazy_and_naive():
    L = import_reference()
    m = small_model(L)
    x, t, y = inputs(2, 64)
    with torch.no_grad():
        ref_lazy = m(x, t, y)
        ref_naive = m(x, t, y, use_lazy=False)
        with integration.install(L):
            ours_lazy = m(x, t, y)
            ours_naive = m(x, t, y, use_lazy=False)
    assert ref_lazy.abs().max() > 0
    assert rel_err(ours_lazy, ref_lazy) < 1e-5
    assert rel_err(ours_naive, ref_naive) < 1e-5
    assert rel_err(ours_lazy, ours_naive) < 1e-5  # lazy == naive through the new kernels


def test_small_model_backward_fp32():
    L = import_reference()
    m = small_model(L)
    x, t, y = inputs(2, 64, seed=1)
    names = [n for n, _ in m.named_parameters() if n.endswith(("read_logits", "write_weight"))]
    params = dict(m.named_parameters())

    def grads():
        m.zero_grad(set_to_none=True)
        xr = x.clone().requires_grad_(True)
        out = m(xr, t, y)
        (out * torch.linspace(-1, 1, out.numel(), device="cuda").view_as(out)).sum().backward()
        return [params[n].grad.clone() for n in names] + [xr.grad.clone()]

    ref = grads()
    with integration.install(L):
        ours = grads()
    for n, a, b in zip(names + ["x"], ours, ref):
        assert rel_err(a, b) < 1e-4, n


def test_released_b4_model_bf16_autocast():
    L = import_reference()
    from flowmatching_lthc.models import build_model

    torch.manual_seed(0)
    m = build_model("lthc_b4_velocity").cuda()
    reseed(m, 2)
    x, t, y = inputs(2, 256, seed=2)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        try:
            ref = m(x, t, y)  # the reference's eager code + its Triton materialise op
        except Exception as e:  # the reference's own Triton path, not ours
            pytest.skip(f"reference Triton path unavailable here: {type(e).__name__}: {e}")
        with integration.install(L):
            ours = m(x, t, y)
    assert ref.abs().max() > 0
    assert rel_err(ours, ref) < 2e-2


def test_triton_materialise_comparator_parity():
    """Our materialisation vs jit_thc::final_accumulate_b4_12_traceable on the same B/4 inputs."""
    import_reference()
    cfg = workloads.config2(B=4, device="cuda", seed=3)
    from flowmatching_lthc_b200 import ops

    ours = ops.materialise(cfg["x0"], cfg["dz"], cfg["P"])
    try:
        theirs = torch.ops.jit_thc.final_accumulate_b4_12_traceable(cfg["x0"], *cfg["dz"], *cfg["P"])
    except Exception as e:
        pytest.skip(f"reference Triton op unavailable here: {type(e).__name__}: {e}")
    assert rel_err(ours, theirs) < 2e-2


def test_doubled_batch_sampler_matches_the_reference_sampler():
    """sample_heun with one [cond; uncond] forward per step gives the reference's
    two-call CFG Heun result (same noise), with and without the new kernels."""
    L = import_reference()
    from flowmatching_lthc.sampling import sample_heun as reference_sample

    from flowmatching_lthc_b200.sampling import sample_heun

    m = small_model(L).eval()
    labels = torch.tensor([1, 5, 999], device="cuda")
    kw = dict(image_size=64, steps=4, cfg_scale=1.5, interval=(0.1, 1.0), prediction="velocity")
    torch.manual_seed(3)
    ref = reference_sample(m, labels, **kw)
    torch.manual_seed(3)
    ours = sample_heun(m, labels, **kw)
    assert ref.abs().max() > 0
    assert rel_err(ours, ref) < 1e-4
    with integration.install(L):
        torch.manual_seed(3)
        ours_kernels = sample_heun(m, labels, **kw)
    assert rel_err(ours_kernels, ref) < 1e-4
