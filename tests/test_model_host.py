"""CPU tests of the standalone model's host-side contract: the released model's
checkpoint keys and shapes (recorded from the reference's build_model by
tests/golden/make_model_golden.py), legacy key migration, the seeded weight fill
the parity fixtures rely on, and the loud failure on CPU tensors (no fallback)."""
from __future__ import annotations

import json

import pytest
import torch

from conftest import GOLDEN, import_reference
from flowmatching_lthc_b200 import model as M


def test_b4_state_dict_matches_the_reference_checkpoint_layout():
    want = json.loads((GOLDEN / "b4_state_dict_keys.json").read_text())
    m = M.build_model("lthc_b4_velocity")
    got = {k: list(v.shape) for k, v in m.state_dict().items()}
    assert list(got) == list(want)  # same keys in the same order
    assert got == want
    assert sum(v.numel() for v in m.state_dict().values()) == 91_633_968


def test_b4_defaults_and_names():
    for name in M.MODEL_NAMES:
        m = M.build_model(name, depth=1)
        assert (m.hidden_size, m.num_heads, m.patch_size, m.workspace_grid, m.high_grid) == (768, 12, 4, 16, 64)
    with pytest.raises(ValueError, match="unknown model"):
        M.build_model("local_thc_v2_fused_final12_shared_adaln_b4")
    assert M.SharedReadFusedFinal12LocalTHCSharedAdaLNJiT is M.LTHCModel


def test_fresh_model_has_the_reference_initialisation():
    m = M.LTHCModel(input_size=64, hidden_size=64, depth=2, num_heads=4, bottleneck_dim=32, workspace_grid=4,
                    num_classes=10)
    assert torch.count_nonzero(m.final_layer.linear.weight) == 0
    assert torch.count_nonzero(m.shared_adaLN_modulation[1].weight) == 0
    assert torch.count_nonzero(m.shared_read.read_logits) == 0
    assert bool((m.blocks[0].write.write_weight == 1).all())
    assert torch.count_nonzero(m.blocks[0].branch.attn.qkv.bias) == 0
    assert 0.015 < m.y_embedder.embedding_table.weight.std().item() < 0.025


def test_legacy_checkpoint_keys_are_migrated():
    m = M.LTHCModel(input_size=64, hidden_size=64, depth=2, num_heads=4, bottleneck_dim=32, workspace_grid=4,
                    num_classes=10)
    M.fill_seeded_(m, 9)
    sd = m.state_dict()
    legacy = {}
    for k, v in sd.items():
        k = k.replace("shared_read.read_logits", "shared_write.write_logits")
        k = k.replace(".write.write_weight", ".read.read_weight")
        legacy[k] = v.clone()
    assert "shared_write.write_logits" in legacy and "blocks.1.read.read_weight" in legacy
    m2 = M.LTHCModel(input_size=64, hidden_size=64, depth=2, num_heads=4, bottleneck_dim=32, workspace_grid=4,
                     num_classes=10)
    m2.load_state_dict(legacy)
    for k, v in m2.state_dict().items():
        assert torch.equal(v, sd[k]), k


def test_seeded_fill_is_a_function_of_seed_and_name():
    kw = dict(input_size=64, hidden_size=64, depth=2, num_heads=4, bottleneck_dim=32, workspace_grid=4, num_classes=10)
    a, b = M.fill_seeded_(M.LTHCModel(**kw), 3), M.fill_seeded_(M.LTHCModel(**kw), 3)
    c = M.fill_seeded_(M.LTHCModel(**kw), 4)
    for (k, va), vb, vc in zip(a.state_dict().items(), b.state_dict().values(), c.state_dict().values()):
        assert torch.equal(va, vb), k
        assert not torch.equal(va, vc), k


def test_seeded_fill_gives_the_reference_model_identical_weights():
    L = import_reference()
    kw = dict(input_size=64, patch_size=4, hidden_size=64, depth=12, num_heads=4, bottleneck_dim=32, workspace_grid=4,
              num_classes=10)
    ref = M.fill_seeded_(L.SharedReadFusedFinal12LocalTHCSharedAdaLNJiT(**kw, pool_groups=64), 3)
    ours = M.fill_seeded_(M.LTHCModel(**kw), 3)
    rs, os_ = ref.state_dict(), ours.state_dict()
    assert list(rs) == list(os_)
    for k in rs:
        assert torch.equal(rs[k], os_[k]), k
    # the checkpoint of one loads into the other
    M.LTHCModel(**kw).load_state_dict(rs)


def test_cpu_forward_raises_instead_of_falling_back():
    m = M.LTHCModel(input_size=64, hidden_size=64, depth=2, num_heads=4, bottleneck_dim=32, workspace_grid=4,
                    num_classes=10)
    x, t, y = torch.randn(1, 3, 64, 64), torch.rand(1), torch.tensor([1])
    # the LTHC operators have no CPU kernel: the dispatcher refuses CPU tensors
    with pytest.raises(NotImplementedError, match="lthc_b200"):
        m(x, t, y)
    with pytest.raises(NotImplementedError, match="lthc_b200"):
        m(x, t, y, use_lazy=False)


def test_image_noise_does_not_depend_on_sharding():
    from flowmatching_lthc_b200.sampling import image_noise

    full = image_noise(5, 0, 6, image_size=8)
    parts = torch.cat([image_noise(5, 0, 2, image_size=8), image_noise(5, 2, 5, image_size=8),
                       image_noise(5, 5, 6, image_size=8)])
    assert torch.equal(full, parts)
    assert abs(full.mean().item()) < 0.2 and 0.8 < full.std().item() < 1.2
