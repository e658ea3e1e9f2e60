"""Host-side behaviour of the PyTorch operator layer and the drop-in installer:
schemas, fake (meta) shapes for torch.compile, shape errors, the loud failure
on CPU tensors, and install/uninstall on the reference model.  CPU only."""
from __future__ import annotations

import pytest
import torch

import flowmatching_lthc_b200 as F
from conftest import import_reference
from flowmatching_lthc_b200 import integration, modules, ops


def meta(*shape, dtype=torch.bfloat16):
    return torch.empty(*shape, device="meta", dtype=dtype)


def test_fake_shapes():
    x = meta(2, 64, 64, 768)
    a = meta(768, 16, dtype=torch.float32)
    assert torch.ops.lthc_b200.read(x, a).shape == (2, 256, 768)
    dz = [meta(2, 256, 768) for _ in range(12)]
    be = [meta(768, 16, dtype=torch.float32) for _ in range(12)]
    assert torch.ops.lthc_b200.materialise(x, dz, be).shape == (2, 64, 64, 768)
    gdz, gb = torch.ops.lthc_b200.materialise_bwd(x, dz, be, True, True)
    assert len(gdz) == 12 and gdz[0].shape == (2, 256, 768) and gb.shape == (12, 768, 16)
    assert torch.ops.lthc_b200.write(dz[0], be[0]).shape == (2, 64, 64, 768)
    assert torch.ops.lthc_b200.lazy_update(dz[0], dz[1], be[0], be[1]).shape == (2, 256, 768)
    assert torch.ops.lthc_b200.weight_grad(x, dz[:3]).shape == (3, 768, 16)
    gx, ga = torch.ops.lthc_b200.read_bwd(x, dz[0], a, True, True, x)
    assert gx.shape == x.shape and ga.shape == (768, 16)
    gdz = torch.ops.lthc_b200.materialise_grad_dz(x, be)
    assert len(gdz) == 12 and gdz[0].shape == (2, 256, 768)
    assert torch.ops.lthc_b200.materialise_grad_beta(x, dz).shape == (12, 768, 16)
    assert ops.final_accumulate_b4_12_grad_dz_ptr_traceable(x, *be).shape == (12, 2, 256, 768)
    assert ops.final_accumulate_b4_12_grad_beta_ptr_traceable(x, *dz).shape == (12, 768, 16)


def test_cpu_tensors_fail_loudly():
    with pytest.raises(NotImplementedError):
        F.read(torch.zeros(1, 8, 8, 8), torch.zeros(8, 16))
    with pytest.raises(NotImplementedError):
        F.materialise(torch.zeros(1, 8, 8, 8), [torch.zeros(1, 4, 8)], [torch.zeros(8, 16)])


def test_module_geometry_and_shape_errors():
    with pytest.raises(ValueError):
        modules.SharedLocalRead(64, 8, 768, 768)  # 8x8 cells are not implemented
    r = modules.SharedLocalRead(64, 16, 768, 768)
    with pytest.raises(ValueError, match=r"expected \[B,64,64,768\]"):
        r.read(torch.zeros(1, 32, 32, 768))
    w = modules.LayerLocalWrite(64, 16, 768, 768)
    with pytest.raises(ValueError, match=r"expected \[B,256,768\]"):
        w.write(torch.zeros(1, 255, 768))
    assert dict(r.named_parameters())["read_logits"].shape == (768, 16)
    assert dict(w.named_parameters())["write_weight"].shape == (768, 16)


def test_group_weights_expand_per_channel():
    w = torch.arange(3 * 16, dtype=torch.float32).view(3, 16)
    e = modules.per_channel(w, 12)
    assert e.shape == (12, 16) and torch.equal(e[4], w[1])


def test_install_and_uninstall_on_the_reference():
    L = import_reference()
    originals = {(c, m): getattr(L, c).__dict__.get(m) for c, m, _ in integration.PATCHES}
    keys_before = list(L.SharedReadFusedFinal12LocalTHCSharedAdaLNJiT(depth=12).state_dict().keys())
    with integration.install(L):
        for c, m, fn in integration.PATCHES:
            assert getattr(L, c).__dict__[m] is fn
        model = L.SharedReadFusedFinal12LocalTHCSharedAdaLNJiT(depth=12)
        assert list(model.state_dict().keys()) == keys_before
        with pytest.raises(NotImplementedError):  # CPU tensors are refused, not silently computed
            model.shared_read.read(torch.zeros(1, 64, 64, 768))
    for (c, m), fn in originals.items():
        assert getattr(L, c).__dict__.get(m) is fn


def test_reference_op_mirrors_exist():
    for name in ["final_accumulate_b4_12_traceable", "final_accumulate_b4_traceable",
                 "final_accumulate_b4_12_grad_dz_ptr_traceable", "final_accumulate_b4_12_grad_beta_ptr_traceable",
                 "local_write_traceable", "local_read_traceable", "local_read_add_traceable",
                 "local_weight_grad_traceable"]:
        assert callable(getattr(ops, name))
    with pytest.raises(ValueError):
        ops.final_accumulate_b4_12_traceable(torch.zeros(1), torch.zeros(1))


def test_call_routes_meta_and_cpu_tensors_through_the_dispatcher():
    """ops.call takes the direct CUDA path only for real CUDA tensors without an
    autograd graph; meta tensors get the registered fake implementation and CPU
    tensors the operator's own error."""
    m = torch.empty(2, 64, 768, device="meta", dtype=torch.bfloat16)
    w = torch.empty(768, 16, device="meta", dtype=torch.bfloat16)
    out = ops.call(ops.lazy_update, m, m, w, w)
    assert out.device.type == "meta" and out.shape == m.shape
    c = torch.zeros(2, 64, 768, dtype=torch.bfloat16)
    wc = torch.zeros(768, 16, dtype=torch.bfloat16)
    with pytest.raises((ValueError, NotImplementedError)):
        ops.call(ops.lazy_update, c, c, wc, wc)
