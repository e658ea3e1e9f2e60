"""Patch embedding fused with the shared read on the tensor cores
(BottleneckPatchEmbedNHWC.forward + SharedLocalRead.read, local_thc.py:64-89,
1211-1223), through the operator layer / C ABI.

X0 is checked against the same computation in torch on the same bf16 operands
(fp32 accumulation, the convolution rounded to bf16 before the bias add as in
the reference; the tensor cores accumulate in another order, so a bf16 rounding
can move by one ulp: > 99 % of X0 identical, max difference 2e-2 of the largest
magnitude) and against the reference's own module under bf16 autocast (cuDNN:
> 99.9 % identical, 2e-2).  Z must equal lthc_read_fwd applied to the X0 the kernel wrote,
bit for bit (same fp32 FMA order).
"""
from __future__ import annotations

import pytest
import torch

from conftest import import_reference
from flowmatching_lthc_b200 import ops

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def rel_err(a, b) -> float:
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def exact_fraction(a, b) -> float:
    return (a.detach().cpu() == b.detach().cpu()).float().mean().item()


def make(B, cin, H, C, seed, img_dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    img = torch.randn(B, cin, 4 * H, 4 * H, generator=g).to(img_dtype).cuda()
    w1 = (torch.randn(128, cin, 4, 4, generator=g) * (1.0 / (cin * 16) ** 0.5)).cuda()
    w2 = (torch.randn(C, 128, 1, 1, generator=g) * (1.0 / 128 ** 0.5)).cuda()
    b2 = (torch.randn(C, generator=g) * 0.1).cuda()
    alpha = torch.softmax(torch.randn(C, 16, generator=g), -1).to(BF).cuda()
    return img, w1, w2, b2, alpha


def emulate(img, w1, w2, b2):
    """The two convolutions in torch on the bf16-cast operands, fp32 accumulation."""
    b, cin, s, _ = img.shape
    h = s // 4
    patches = img.to(BF).reshape(b, cin, h, 4, h, 4).permute(0, 2, 4, 1, 3, 5).reshape(-1, cin * 16).float()
    h1 = (patches @ w1.to(BF).reshape(128, -1).float().t()).to(BF)
    conv = (h1.float() @ w2.to(BF).reshape(w2.shape[0], 128).float().t()).to(BF)
    x0 = (conv.float() + b2.to(BF).float()).to(BF)  # the bias is a separate bf16 add
    return x0.reshape(b, h, h, -1)


@pytest.mark.parametrize("B, cin, H, C", [(2, 3, 64, 768), (3, 3, 64, 256), (1, 1, 32, 512), (2, 4, 32, 256),
                                          (1, 2, 96, 768)])
def test_matches_torch_on_bf16_operands_and_read(B, cin, H, C):
    img, w1, w2, b2, alpha = make(B, cin, H, C, seed=B * 100 + cin * 10 + H + C)
    x0, z = ops.patch_embed_read(img, w1, w2, b2, alpha)
    ref = emulate(img, w1, w2, b2)
    assert x0.shape == ref.shape and x0.dtype == BF
    assert exact_fraction(x0, ref) > 0.99
    assert rel_err(x0, ref) < 2e-2
    zr = ops.read(x0, alpha)
    assert torch.equal(z, zr)


def test_bf16_image_input():
    img, w1, w2, b2, alpha = make(2, 3, 64, 768, seed=7, img_dtype=BF)
    x0, z = ops.patch_embed_read(img, w1, w2, b2, alpha)
    assert exact_fraction(x0, emulate(img, w1, w2, b2)) > 0.99
    assert torch.equal(z, ops.read(x0, alpha))


def test_matches_reference_module_under_autocast():
    L = import_reference()
    torch.manual_seed(0)
    emb = L.BottleneckPatchEmbedNHWC(256, 4, 3, 128, 768).cuda()
    img = torch.randn(4, 3, 256, 256, device="cuda")
    alpha = torch.softmax(torch.randn(768, 16, device="cuda"), -1).to(BF)
    with torch.no_grad(), torch.autocast("cuda", dtype=BF):
        ref = emb(img)
    x0, z = ops.patch_embed_read(img, emb.proj1.weight, emb.proj2.weight, emb.proj2.bias, alpha)
    assert ref.dtype == BF
    assert rel_err(x0, ref) < 2e-2
    assert exact_fraction(x0, ref) > 0.999
    assert rel_err(z, ops.read(ref, alpha)) < 2e-2


def test_autograd_matches_reference():
    """Gradients of the fused op (read backward + the convolutions' backward as
    library GEMMs) against autograd through the reference module and the read."""
    L = import_reference()
    torch.manual_seed(1)
    emb = L.BottleneckPatchEmbedNHWC(128, 4, 3, 128, 256).cuda()
    img = torch.randn(2, 3, 128, 128, device="cuda")
    logits = torch.randn(256, 16, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(2)
    gx0 = torch.randn(2, 32, 32, 256, device="cuda", generator=g).to(BF)
    gz = torch.randn(2, 64, 256, device="cuda", generator=g).to(BF)

    def run(fused: bool):
        emb.zero_grad(set_to_none=True)
        lg = logits.clone().requires_grad_(True)
        with torch.autocast("cuda", dtype=BF):
            alpha = torch.softmax(lg, -1).to(BF)
            if fused:
                x0, z = ops.patch_embed_read(img, emb.proj1.weight, emb.proj2.weight, emb.proj2.bias, alpha)
            else:
                x0 = emb(img)
                z = ops.read(x0, alpha)
        ((x0.float() * gx0.float()).sum() + (z.float() * gz.float()).sum()).backward()
        return [emb.proj1.weight.grad.clone(), emb.proj2.weight.grad.clone(), emb.proj2.bias.grad.clone(),
                lg.grad.clone()]

    for a, b in zip(run(True), run(False)):
        assert rel_err(a, b) < 3e-2


def test_validation():
    img, w1, w2, b2, alpha = make(1, 3, 64, 768, seed=3)
    with pytest.raises(ValueError):
        ops.patch_embed_read(img, w1, w2[:700], b2[:700], alpha[:700])   # C not a multiple of 256
    with pytest.raises(ValueError):
        ops.patch_embed_read(img[:, :, :200, :200], w1, w2, b2, alpha)  # grid side not a multiple of 32
    assert not ops.embed_supported(img, w1[:, :, :2], w2)
