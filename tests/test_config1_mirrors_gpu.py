"""BASELINE configuration 1 exactly on the GPU, and every mirror of the reference's
jit_thc op surface (ops.py) called on the GPU.

Configuration 1 (local_thc.py:1211-1276): B = 2, 16x16 workspace, C = 768, fp32,
seed 0, the read weights R ~ N(1/16, 0.01) used directly as alpha.  The read,
write and write_add kernels must equal the C oracle bit for bit on the full
inputs and the reference's own outputs (tests/golden/config1_b2_c768_f32.pt, made
by tests/golden/make_golden.py config1; the residual-sized outputs as a fixed
sample) within 1e-5 relative.

Mirrors (local_thc_triton_kernels.py:1578-1598, 1669-1736, 1800-1894, 2673-2764)
at L = 12, B = 2, C = 128, bf16: outputs equal the oracle bit for bit (the
tensor-core grad_dz within one unit in the last place), weight gradients within
1e-5 relative (they sum in another order)."""
from __future__ import annotations

import pytest
import torch

from conftest import GOLDEN, close_16bit
from flowmatching_lthc_b200 import ops
from flowmatching_lthc_b200 import workloads as W
from oracle import lthc_oracle as O

pytestmark = pytest.mark.gpu
RTOL = 1e-5


def rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def bits_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    a, b = a.detach().cpu().contiguous(), b.detach().cpu().contiguous()
    return a.dtype == b.dtype and a.shape == b.shape and torch.equal(a.view(torch.uint8), b.view(torch.uint8))


def test_baseline_config1_read_write_and_write_add():
    gold = torch.load(GOLDEN / "config1_b2_c768_f32.pt")
    cpu = W.config1()
    assert (cpu["B"], cpu["G"], cpu["C"]) == (2, 16, 768) and cpu["x"].dtype == torch.float32
    dev = {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in cpu.items()}
    z = ops.read(dev["x"], dev["R"])
    assert bits_equal(z, O.read(cpu["x"], cpu["R"]))
    assert rel(z, gold["read_z"]) < RTOL
    stride = gold["meta"]["sample_stride"]
    wa = ops.write_add(dev["x"], dev["dz"], dev["P"])
    assert bits_equal(wa, O.write_add(cpu["x"], cpu["dz"], cpu["P"]))
    assert rel(wa.reshape(-1)[::stride], gold["write_add_sample"]) < RTOL
    w = ops.write(dev["dz"], dev["P"])
    assert bits_equal(w, O.write(cpu["dz"], cpu["P"]))
    assert rel(w.reshape(-1)[::stride], gold["write_sample"]) < RTOL


def _mirror_inputs():
    g = torch.Generator().manual_seed(41)
    B, G, C, L = 2, 16, 128, 12
    bf = torch.bfloat16
    x0 = torch.randn(B, 4 * G, 4 * G, C, generator=g).to(bf)
    gout = torch.randn(B, 4 * G, 4 * G, C, generator=g).to(bf)
    dz = [(0.1 * torch.randn(B, G * G, C, generator=g)).to(bf) for _ in range(L)]
    P = [0.02 * torch.randn(C, 16, generator=g) for _ in range(L)]
    alpha = torch.softmax(torch.randn(C, 16, generator=g), -1).to(bf)
    return x0, gout, dz, P, alpha


def test_final_accumulate_mirrors():
    x0, gout, dz, P, _ = _mirror_inputs()
    want = O.materialise(x0, dz, P)
    dzd, Pd = [t.cuda() for t in dz], [p.cuda() for p in P]
    out12 = ops.final_accumulate_b4_12_traceable(x0.cuda(), *dzd, *Pd)
    assert bits_equal(out12, want)
    out = ops.final_accumulate_b4_traceable(x0.cuda(), torch.stack(dzd), torch.stack(Pd))
    assert bits_equal(out, want)
    with pytest.raises(ValueError, match="12 dz and 12 beta"):
        ops.final_accumulate_b4_12_traceable(x0.cuda(), *dzd[:11], *Pd)


def test_final_accumulate_grad_mirrors_need_no_dummy_inputs():
    """grad_dz from the betas alone and grad_beta from the updates alone, each equal
    to the fused backward and to the oracle."""
    _, gout, dz, P, _ = _mirror_inputs()
    rdz, rb = O.materialise_bwd(gout, dz, P)
    g, dzd, Pd = gout.cuda(), [t.cuda() for t in dz], [p.cuda() for p in P]
    gdz = ops.final_accumulate_b4_12_grad_dz_ptr_traceable(g, *Pd)
    assert gdz.shape == (12, 2, 256, 128)
    assert ops.materialise_bwd_uses_tensor_cores(2, 16, 128, 12, torch.bfloat16)
    for l in range(12):
        assert close_16bit(gdz[l], rdz[l]), l
    gb = ops.final_accumulate_b4_12_grad_beta_ptr_traceable(g, *dzd)
    assert gb.dtype == torch.float32 and gb.shape == (12, 128, 16)
    assert rel(gb, rb) < RTOL
    fused_dz, fused_b = ops.materialise_bwd(g, dzd, Pd, True, True)
    assert all(torch.equal(a, b) for a, b in zip(fused_dz, gdz.unbind(0)))
    assert torch.equal(fused_b, gb)  # same kernels, same fixed reduction order


def test_local_read_write_mirrors():
    """Legacy naming of the reference's Triton read/write ops: local_write = read,
    local_read = write, local_read_add(z, w, x) = x + write(z)."""
    x0, gout, dz, P, alpha = _mirror_inputs()
    beta = P[0].to(torch.bfloat16)
    z = ops.local_write_traceable(x0.cuda(), alpha.cuda())
    assert bits_equal(z, O.read(x0, alpha))
    w = ops.local_read_traceable(dz[0].cuda(), beta.cuda())
    assert bits_equal(w, O.write(dz[0], beta))
    wa = ops.local_read_add_traceable(dz[0].cuda(), beta.cuda(), x0.cuda())
    assert bits_equal(wa, O.write_add(x0, dz[0], beta))
    gw = ops.local_weight_grad_traceable(gout.cuda(), dz[3].cuda())
    assert gw.shape == (128, 16) and gw.dtype == torch.float32
    assert rel(gw, O.weight_grad(gout, [dz[3]])[0]) < RTOL
