"""The CUDA-graph training step (flowmatching_lthc_b200.training) against the same
step run eagerly: identical weights, inputs and optimizer, so the losses and the
updated parameters must agree bit for bit after several steps (the replays launch
the same kernels in the same order)."""
from __future__ import annotations

import pytest
import torch

from flowmatching_lthc_b200 import dist as D
from flowmatching_lthc_b200 import model as M
from flowmatching_lthc_b200.training import GraphedTrainStep, flow_matching_step

pytestmark = pytest.mark.gpu

KW = dict(input_size=128, patch_size=4, hidden_size=256, depth=12, num_heads=4, bottleneck_dim=128,
          workspace_grid=8, num_classes=10)


def _setup(seed: int = 5):
    m = M.fill_seeded_(M.LTHCModel(**KW), seed).cuda().train()
    opt = torch.optim.AdamW(m.parameters(), lr=1e-3, fused=True, capturable=True)
    fg = D.FlatGradients(m.parameters())
    return m, opt, fg


def _inputs(B: int = 4):
    g = torch.Generator(device="cuda").manual_seed(9)
    x1 = torch.randn(B, 3, 128, 128, device="cuda", generator=g)
    e = torch.randn(B, 3, 128, 128, device="cuda", generator=g)
    t = torch.rand(B, device="cuda", generator=g)
    y = torch.randint(0, 11, (B,), device="cuda", generator=g)
    tt = t.view(-1, 1, 1, 1)
    zt = tt * x1 + (1 - tt) * e
    v = (x1 - zt) / (1 - tt).clamp_min(0.05)
    return zt, t, y, v


@pytest.mark.parametrize("dtype", [torch.bfloat16, None])
def test_graphed_step_equals_eager_step(dtype):
    zt, t, y, v = _inputs()
    warmup, replays = 2, 3
    m1, opt1, fg1 = _setup()
    l1 = torch.zeros((), device="cuda")
    step1 = flow_matching_step(m1, fg1.zero_grad, zt, t, y, v, l1, dtype)
    losses1 = []
    for _ in range(warmup + replays):
        step1()
        opt1.step()
        losses1.append(l1.item())
    # graphed: its warm-up performs the first `warmup` updates eagerly
    m2, opt2, fg2 = _setup()
    l2 = torch.zeros((), device="cuda")
    graphed = GraphedTrainStep(flow_matching_step(m2, fg2.zero_grad, zt, t, y, v, l2, dtype), opt2.step, warmup)
    losses2 = []
    for _ in range(replays):
        graphed()
        losses2.append(l2.item())
    torch.cuda.synchronize()
    assert losses2 == losses1[warmup:]
    for (n1, p1), (_, p2) in zip(m1.named_parameters(), m2.named_parameters()):
        assert torch.equal(p1, p2), n1


def test_graphed_step_runs_the_exchange_between_the_graphs():
    zt, t, y, v = _inputs()
    m, opt, fg = _setup()
    seen = []
    graphed = GraphedTrainStep(flow_matching_step(m, fg.zero_grad, zt, t, y, v), opt.step, 1)
    graphed(lambda: seen.append(fg.flat.abs().sum().item()))
    assert len(seen) == 1 and seen[0] > 0  # the gradients exist when the exchange runs
    with pytest.raises(ValueError, match="warm-up"):
        GraphedTrainStep(lambda: None, lambda: None, 0)
