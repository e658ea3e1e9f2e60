"""Generates the golden input/output fixtures under tests/golden/ by running the
reference's own eager PyTorch code (tongtongliang/flowmatching_lthc) on CPU.

Run from the repository root with the reference importable, e.g.

    LTHC_REFERENCE=/path/to/flowmatching_lthc python tests/golden/make_golden.py [all|lthc|final|branch|config1]

The reference is only needed to (re)generate the fixtures; the committed ``*.pt``
files are what the tests read.  Every tensor is produced by the reference
functions named below (paths inside the reference repository):

  SharedLocalRead.read / .alpha          flowmatching_lthc/models/local_thc.py:1204-1223
  LayerLocalWrite.write / .write_add     flowmatching_lthc/models/local_thc.py:1261-1276
  LayerLocalWrite.gamma_from_alpha       flowmatching_lthc/models/local_thc.py:1278-1283
  Block.lazy_workspace_update            flowmatching_lthc/models/local_thc.py:1325-1328
  Model.final_accumulate_reference       flowmatching_lthc/models/local_thc.py:1368-1372
  WorkspaceSharedAdaLNBranch.forward (output epilogue), Block.branch_update
                                         flowmatching_lthc/models/local_thc.py:318-323, 1322-1323
  FinalLayerSharedAdaLN (norm_final = RMSNorm, modulate, linear)
                                         flowmatching_lthc/models/local_thc.py:37-38, 865-873
                                         flowmatching_lthc/models/jit_shared_adaln.py:20-30

Gradients come from torch.autograd through the same eager code.  Inputs follow
the distributions of the benchmark configurations (X ~ N(0,1), read weights
~ N(1/16, 0.01) used directly as alpha, write weights ~ N(0, 0.02), workspace
updates ~ N(0,1) or N(0, 0.1)) at sizes small enough to commit.
"""
from __future__ import annotations

import os
import sys
import types
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
if not os.environ.get("LTHC_REFERENCE"):
    sys.exit("set LTHC_REFERENCE to the root of a flowmatching_lthc checkout (the directory that holds "
             "flowmatching_lthc/models/local_thc.py)")
sys.path.insert(0, os.environ["LTHC_REFERENCE"])
sys.dont_write_bytecode = True

from flowmatching_lthc.models import local_thc as L  # noqa: E402


def cell_major_to_nhwc(x: torch.Tensor, g: int) -> torch.Tensor:
    """[B, G*G, 16, C] cell-major -> NHWC [B, 4G, 4G, C] (cell (wy,wx), r = 4*row+col)."""
    b, _, _, c = x.shape
    return x.view(b, g, g, 4, 4, c).permute(0, 1, 3, 2, 4, 5).reshape(b, 4 * g, 4 * g, c).contiguous()


def make_case(name: str, *, B: int, G: int, C: int, dtype: torch.dtype, depth: int, seed: int) -> dict:
    gen = torch.Generator().manual_seed(seed)

    def randn(*shape, mean=0.0, std=1.0):
        return torch.randn(*shape, generator=gen) * std + mean

    hi = 4 * G
    x = cell_major_to_nhwc(randn(B, G * G, 16, C), G).to(dtype)
    R = randn(C, 16, mean=1.0 / 16, std=0.01)
    P = [randn(C, 16, std=0.02) for _ in range(depth)]
    dz = [randn(B, G * G, C).to(dtype) for _ in range(depth)]
    dz_small = [randn(B, G * G, C, std=0.1).to(dtype) for _ in range(depth)]
    g_z = randn(B, G * G, C).to(dtype)
    g_x = randn(B, hi, hi, C).to(dtype)

    read = L.SharedLocalRead(hi, G, C, C, use_softmax_write=False)
    read.read_logits.data.copy_(R)
    writes = []
    for l in range(depth):
        w = L.LayerLocalWrite(hi, G, C, C)
        w.write_weight.data.copy_(P[l])
        writes.append(w)

    out: dict = {"meta": {"name": name, "B": B, "G": G, "C": C, "dtype": str(dtype), "depth": depth, "seed": seed},
                 "x": x, "R": R, "P": torch.stack(P), "dz": torch.stack(dz), "dz_small": torch.stack(dz_small),
                 "g_z": g_z, "g_x": g_x}

    # read (alpha = R directly, cast to the activation dtype as the module does)
    xr = x.clone().requires_grad_(True)
    z = read.read(xr)
    gx, gR = torch.autograd.grad(z, (xr, read.read_logits), g_z)
    out.update(read_z=z.detach(), read_gx=gx, read_gR=gR)

    # write / write_add for layer 0
    d0 = dz[0].clone().requires_grad_(True)
    w0 = writes[0].write(d0)
    gd, gP = torch.autograd.grad(w0, (d0, writes[0].write_weight), g_x)
    out.update(write_out=w0.detach(), write_gdz=gd, write_gP=gP)
    xa = x.clone().requires_grad_(True)
    d0 = dz[0].clone().requires_grad_(True)
    wa = writes[0].write_add(xa, d0)
    gxa, gd, gP = torch.autograd.grad(wa, (xa, d0, writes[0].write_weight), g_x)
    out.update(write_add_out=wa.detach(), write_add_gx=gxa, write_add_gdz=gd, write_add_gP=gP)

    # gamma and the lazy workspace recurrence for layer 0
    block = L.SharedReadLocalTHCSharedAdaLNJiTBlock(C, num_heads=C // 8, high_grid=hi, workspace_grid=G)
    block.write.write_weight.data.copy_(P[0])
    alpha = read.alpha(dtype=dtype)
    out["gamma"] = block.write.gamma_from_alpha(alpha).detach()
    zl = z.detach().clone().requires_grad_(True)
    d0 = dz[0].clone().requires_grad_(True)
    zn = block.lazy_workspace_update(zl, d0, read)
    gzl, gd, gR, gP = torch.autograd.grad(zn, (zl, d0, read.read_logits, block.write.write_weight), g_z)
    out.update(lazy_z=zn.detach(), lazy_gz=gzl, lazy_gdz=gd, lazy_gR=gR, lazy_gP=gP)

    # materialisation over `depth` layers through the pure-torch accumulate loop
    stub = types.SimpleNamespace(blocks=[types.SimpleNamespace(write=w) for w in writes])
    x0 = x.clone().requires_grad_(True)
    dzs = [t.clone().requires_grad_(True) for t in dz_small]
    xl = L.SharedReadLocalTHCSharedAdaLNJiT.final_accumulate_reference(stub, x0, dzs)
    grads = torch.autograd.grad(xl, (x0, *dzs, *[w.write_weight for w in writes]), g_x)
    out.update(mat_out=xl.detach(), mat_gx0=grads[0], mat_gdz=torch.stack(grads[1:1 + depth]),
               mat_gP=torch.stack(grads[1 + depth:]))
    return out


def make_final_case(name: str, *, B: int, T: int, C: int, dtype: torch.dtype, seed: int) -> dict:
    """FinalLayerSharedAdaLN's RMSNorm + modulate (and, in fp32, its whole forward
    including the Linear) with autograd through the same eager code."""
    gen = torch.Generator().manual_seed(seed)

    def randn(*shape, mean=0.0, std=1.0):
        return torch.randn(*shape, generator=gen) * std + mean

    layer = L.FinalLayerSharedAdaLN(C, 4, 3)
    with torch.no_grad():
        layer.norm_final.weight.copy_(randn(C, mean=1.0, std=0.1))
        layer.linear.weight.copy_(randn(48, C, std=0.02))
        layer.linear.bias.copy_(randn(48, std=0.02))
    x = randn(B, T, C).to(dtype)
    t2 = randn(B, 2 * C, std=0.5).to(dtype)
    g_m = randn(B, T, C).to(dtype)
    out: dict = {"meta": {"name": name, "B": B, "T": T, "C": C, "dtype": str(dtype), "seed": seed,
                          "eps": layer.norm_final.eps},
                 "x": x, "t2": t2, "norm_weight": layer.norm_final.weight.detach().clone(), "g_m": g_m,
                 "linear_weight": layer.linear.weight.detach().clone(), "linear_bias": layer.linear.bias.detach().clone()}
    xr = x.clone().requires_grad_(True)
    t2r = t2.clone().requires_grad_(True)
    shift, scale = t2r.chunk(2, dim=1)
    m = L.modulate(layer.norm_final(xr), shift, scale)
    gx, gw, gt2 = torch.autograd.grad(m, (xr, layer.norm_final.weight, t2r), g_m)
    out.update(m=m.detach(), gx=gx, g_norm_weight=gw, g_shift=gt2[:, :C].contiguous(), g_scale=gt2[:, C:].contiguous())
    if dtype == torch.float32:
        out["layer_out"] = layer(x, t2).detach()
    return out


class _Fixed(torch.nn.Module):
    """Stands in for the branch's attention or MLP: returns a fixed leaf tensor so
    the epilogue's inputs (and their gradients) are observable."""

    def __init__(self, value: torch.Tensor) -> None:
        super().__init__()
        self.value = value

    def forward(self, *args):
        return self.value


def make_branch_case(name: str, *, B: int, G: int, C: int, dtype: torch.dtype, seed: int) -> dict:
    """WorkspaceSharedAdaLNBranch.forward's output epilogue (gate product and sum)
    followed by Block.lazy_workspace_update, through the reference's own
    branch_update / lazy_workspace_update with the attention and the MLP replaced
    by fixed leaves A and M and gate_msa = 1, so that dz_attn = A exactly:
        dz = A + gate_mlp (.) M,   z' = z + gamma (.) dz."""
    gen = torch.Generator().manual_seed(seed)

    def randn(*shape, mean=0.0, std=1.0):
        return torch.randn(*shape, generator=gen) * std + mean

    T, hi = G * G, 4 * G
    z = randn(B, T, C).to(dtype)
    A = randn(B, T, C, std=0.5).to(dtype)
    M = randn(B, T, C).to(dtype)
    t6 = randn(B, 6 * C, std=0.5)
    t6[:, 2 * C:3 * C] = 1.0  # gate_msa
    t6 = t6.to(dtype)
    R = randn(C, 16, mean=1.0 / 16, std=0.01)
    P = randn(C, 16, std=0.02)
    g_dz = randn(B, T, C).to(dtype)
    g_zn = randn(B, T, C).to(dtype)

    read = L.SharedLocalRead(hi, G, C, C, use_softmax_write=False)
    read.read_logits.data.copy_(R)
    block = L.SharedReadLocalTHCSharedAdaLNJiTBlock(C, num_heads=C // 8, high_grid=hi, workspace_grid=G)
    block.write.write_weight.data.copy_(P)
    block.branch.to(dtype)
    Ar, Mr = A.clone().requires_grad_(True), M.clone().requires_grad_(True)
    block.branch.attn, block.branch.mlp = _Fixed(Ar), _Fixed(Mr)
    zr, t6r = z.clone().requires_grad_(True), t6.clone().requires_grad_(True)
    dz = block.branch_update(zr, t6r, None)
    zn = block.lazy_workspace_update(zr, dz, read)
    leaves = (zr, Ar, Mr, t6r, read.read_logits, block.write.write_weight)
    g_both = torch.autograd.grad((dz, zn), leaves, (g_dz, g_zn), retain_graph=True)
    g_lazy = torch.autograd.grad(zn, leaves, g_zn)
    out: dict = {"meta": {"name": name, "B": B, "G": G, "C": C, "dtype": str(dtype), "seed": seed},
                 "z": z, "dz_attn": A, "mlp_out": M, "gate": t6[:, 5 * C:].contiguous(), "R": R, "P": P,
                 "g_dz": g_dz, "g_zn": g_zn, "dz": dz.detach(), "z_next": zn.detach()}
    for tag, g in (("both", g_both), ("lazy_only", g_lazy)):
        gz, gA, gM, gt6, gR, gP = g
        out.update({f"{tag}_gz": gz, f"{tag}_gattn": gA, f"{tag}_gmlp": gM,
                    f"{tag}_ggate": gt6[:, 5 * C:].contiguous(), f"{tag}_gR": gR, f"{tag}_gP": gP})
    return out


BRANCH_CASES = [
    ("branch_g4_c768_bf16", dict(B=2, G=4, C=768, dtype=torch.bfloat16, seed=20)),
    ("branch_g4_c40_f32", dict(B=3, G=4, C=40, dtype=torch.float32, seed=21)),
    ("branch_g4_c64_f16", dict(B=2, G=4, C=64, dtype=torch.float16, seed=22)),
]

FINAL_CASES = [
    ("final_t64_c768_bf16", dict(B=2, T=64, C=768, dtype=torch.bfloat16, seed=10)),
    ("final_t16_c40_f32", dict(B=3, T=16, C=40, dtype=torch.float32, seed=11)),
    ("final_t8_c1024_bf16", dict(B=1, T=8, C=1024, dtype=torch.bfloat16, seed=12)),
]

CASES = [
    ("g4_c40_f32", dict(B=2, G=4, C=40, dtype=torch.float32, depth=12, seed=0)),
    ("g4_c40_bf16", dict(B=2, G=4, C=40, dtype=torch.bfloat16, depth=12, seed=1)),
    ("g16_c8_f32", dict(B=1, G=16, C=8, dtype=torch.float32, depth=12, seed=2)),
    ("g2_c64_bf16", dict(B=3, G=2, C=64, dtype=torch.bfloat16, depth=3, seed=3)),
]


# BASELINE configuration 1 exactly (B = 2, 16x16 workspace, C = 768, fp32, R used as
# alpha without the softmax, seed 0), inputs from flowmatching_lthc_b200.workloads.config1.
# The residual-sized outputs are 25 MB each, so a fixed sample of positions is kept.
CONFIG1_SAMPLE_STRIDE = 97


def make_config1_case(name: str) -> dict:
    sys.path.insert(0, str(HERE.parent.parent))
    from flowmatching_lthc_b200 import workloads as W

    cfg = W.config1()
    B, G, C = cfg["B"], cfg["G"], cfg["C"]
    hi = 4 * G
    read = L.SharedLocalRead(hi, G, C, C, use_softmax_write=False)
    read.read_logits.data.copy_(cfg["R"])
    write = L.LayerLocalWrite(hi, G, C, C)
    write.write_weight.data.copy_(cfg["P"])
    with torch.no_grad():
        z = read.read(cfg["x"])
        wa = write.write_add(cfg["x"], cfg["dz"])
        w = write.write(cfg["dz"])
    idx = torch.arange(0, wa.numel(), CONFIG1_SAMPLE_STRIDE)
    return {"meta": {"name": name, "B": B, "G": G, "C": C, "dtype": "torch.float32", "seed": 0,
                     "sample_stride": CONFIG1_SAMPLE_STRIDE},
            "read_z": z, "write_add_sample": wa.reshape(-1)[idx].clone(), "write_sample": w.reshape(-1)[idx].clone(),
            "write_add_sum": wa.double().sum().item(), "read_z_sum": z.double().sum().item()}


def main(which: str = "all") -> None:
    jobs = []
    if which in ("all", "config1"):
        jobs += [("config1_b2_c768_f32", lambda name: make_config1_case(name), {})]
    if which in ("all", "lthc"):
        jobs += [(name, make_case, kw) for name, kw in CASES]
    if which in ("all", "final"):
        jobs += [(name, make_final_case, kw) for name, kw in FINAL_CASES]
    if which in ("all", "branch"):
        jobs += [(name, make_branch_case, kw) for name, kw in BRANCH_CASES]
    for name, fn, kw in jobs:
        case = fn(name, **kw)
        path = HERE / f"{name}.pt"
        torch.save(case, path)
        print(f"wrote {path} ({path.stat().st_size} bytes)")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "all")
