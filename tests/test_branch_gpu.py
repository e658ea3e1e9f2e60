"""The workspace branch's output epilogue fused with the lazy update
(WorkspaceSharedAdaLNBranch.forward's gate product and sum, local_thc.py:318-323,
then lazy_workspace_update, :1325-1328) through the operator layer / C ABI.

Elementwise outputs (dz, z', grad dz_attn, grad mlp_out) are bit-exact against
the C oracle, which rounds in the same order; the reductions (grad gate over an
image's rows, grad alpha / beta over all rows) are fp32 sums in another order:
1e-5 relative.  dz also equals the reference's eager expression bit for bit,
and z' equals the unfused lazy_update applied to that dz bit for bit.
"""
from __future__ import annotations

import pytest
import torch

from conftest import GOLDEN
from flowmatching_lthc_b200 import ops
from oracle import lthc_oracle as O

pytestmark = pytest.mark.gpu
DTYPES = [torch.float32, torch.bfloat16, torch.float16]
TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 5e-3}


def rel_err(a, b) -> float:
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def make(B, T, C, dtype, seed, gate_in_t6=False):
    g = torch.Generator().manual_seed(seed)
    z = torch.randn(B, T, C, generator=g).to(dtype)
    attn = (torch.randn(B, T, C, generator=g) * 0.5).to(dtype)
    mlp = torch.randn(B, T, C, generator=g).to(dtype)
    t6 = (torch.randn(B, 6 * C, generator=g) * 0.5).to(dtype)
    alpha = (torch.randn(C, 16, generator=g) * 0.01 + 1 / 16).to(dtype)
    beta = (torch.randn(C, 16, generator=g) * 0.02).to(dtype)
    gd = torch.randn(B, T, C, generator=g).to(dtype)
    gz = torch.randn(B, T, C, generator=g).to(dtype)
    cpu = dict(z=z, attn=attn, mlp=mlp, gate=t6[:, 5 * C:].contiguous(), alpha=alpha, beta=beta, gd=gd, gz=gz)
    dev = {k: v.cuda() for k, v in cpu.items()}
    if gate_in_t6:
        dev["gate"] = t6.cuda().chunk(6, dim=-1)[5]  # a strided view, as the model passes it
    return cpu, dev


SHAPES = [(2, 256, 768), (1, 16, 40), (3, 37, 64), (5, 1, 8), (64, 256, 768), (1, 4096, 1024)]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("B, T, C", SHAPES)
def test_forward_matches_oracle(B, T, C, dtype):
    cpu, dev = make(B, T, C, dtype, seed=B * 7 + T + C)
    dz, zn = ops.branch_lazy_update(dev["z"], dev["attn"], dev["mlp"], dev["gate"], dev["alpha"], dev["beta"])
    rdz, rzn = O.branch_fwd(cpu["z"], cpu["attn"], cpu["mlp"], cpu["gate"], cpu["alpha"], cpu["beta"])
    assert torch.equal(dz.cpu(), rdz)
    assert torch.equal(zn.cpu(), rzn)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("with_gdz", [True, False])
@pytest.mark.parametrize("B, T, C", SHAPES)
def test_backward_matches_oracle(B, T, C, dtype, with_gdz):
    cpu, dev = make(B, T, C, dtype, seed=B * 5 + T + C + with_gdz)
    dz, _ = O.branch_fwd(cpu["z"], cpu["attn"], cpu["mlp"], cpu["gate"], cpu["alpha"], cpu["beta"])
    ref = O.branch_bwd(cpu["gd"] if with_gdz else None, cpu["gz"], dz, cpu["mlp"], cpu["gate"], cpu["alpha"],
                       cpu["beta"])
    ours = ops.branch_lazy_update_bwd(dev["gd"] if with_gdz else None, dev["gz"], dz.cuda(), dev["mlp"], dev["gate"],
                                      dev["alpha"], dev["beta"])
    assert torch.equal(ours[0].cpu(), ref[0])  # grad dz_attn
    assert torch.equal(ours[1].cpu(), ref[1])  # grad mlp_out
    for a, b in zip(ours[2:], ref[2:]):        # grad gate, grad alpha, grad beta (fp32 sums)
        assert rel_err(a, b) < 1e-5


@pytest.mark.parametrize("dtype", DTYPES)
def test_equals_reference_expression_and_unfused_lazy(dtype):
    _, d = make(4, 256, 768, dtype, seed=3, gate_in_t6=True)
    dz, zn = ops.branch_lazy_update(d["z"], d["attn"], d["mlp"], d["gate"], d["alpha"], d["beta"])
    eager = d["attn"] + d["gate"].unsqueeze(1) * d["mlp"]  # local_thc.py:321-323
    assert torch.equal(dz, eager)
    assert torch.equal(zn, ops.lazy_update(d["z"], eager, d["alpha"], d["beta"]))


def test_strided_gate_view_equals_contiguous():
    _, d = make(3, 64, 256, torch.bfloat16, seed=4, gate_in_t6=True)
    assert not d["gate"].is_contiguous()
    a = ops.branch_lazy_update(d["z"], d["attn"], d["mlp"], d["gate"], d["alpha"], d["beta"])
    b = ops.branch_lazy_update(d["z"], d["attn"], d["mlp"], d["gate"].contiguous(), d["alpha"], d["beta"])
    assert all(torch.equal(x, y) for x, y in zip(a, b))


@pytest.mark.parametrize("name", ["branch_g4_c768_bf16", "branch_g4_c40_f32", "branch_g4_c64_f16"])
def test_golden_fixtures(name):
    """Against the reference's own branch_update / lazy_workspace_update outputs."""
    c = torch.load(GOLDEN / f"{name}.pt")
    dt = c["z"].dtype
    cu = lambda t: t.cuda()  # noqa: E731
    a, p = cu(c["R"].to(dt)), cu(c["P"].to(dt))
    dz, zn = ops.branch_lazy_update(cu(c["z"]), cu(c["dz_attn"]), cu(c["mlp_out"]), cu(c["gate"]), a, p)
    assert torch.equal(dz.cpu(), c["dz"])
    assert rel_err(zn, c["z_next"]) < TOL[dt]
    for tag, gd in (("both", cu(c["g_dz"])), ("lazy_only", None)):
        g_attn, g_mlp, g_gate, ga, gb = ops.branch_lazy_update_bwd(gd, cu(c["g_zn"]), dz, cu(c["mlp_out"]),
                                                                    cu(c["gate"]), a, p)
        assert rel_err(g_attn, c[f"{tag}_gattn"]) < TOL[dt]
        assert rel_err(g_mlp, c[f"{tag}_gmlp"]) < TOL[dt]
        assert rel_err(g_gate.to(dt), c[f"{tag}_ggate"]) < TOL[dt]
        assert rel_err(ga, c[f"{tag}_gR"]) < TOL[dt]
        assert rel_err(gb, c[f"{tag}_gP"]) < TOL[dt]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_autograd_matches_eager(dtype):
    """Gradients through the registered autograd formula against torch autograd of
    the eager expression (both outputs used, as in the model: dz feeds the
    materialisation, z' the next block)."""
    _, d = make(2, 256, 768, dtype, seed=5)
    g = torch.Generator(device="cuda").manual_seed(6)
    w_dz = torch.randn(d["z"].shape, device="cuda", generator=g).to(dtype)
    w_zn = torch.randn(d["z"].shape, device="cuda", generator=g).to(dtype)

    def run(fused: bool):
        leaves = [d[k].clone().requires_grad_(True) for k in ("z", "attn", "mlp", "gate", "alpha", "beta")]
        z, attn, mlp, gate, alpha, beta = leaves
        if fused:
            dz, zn = ops.branch_lazy_update(z, attn, mlp, gate, alpha, beta)
        else:
            dz = attn + gate.unsqueeze(1) * mlp
            zn = z + (alpha.float() * beta.float()).sum(-1).to(dtype) * dz
        ((dz.float() * w_dz.float()).sum() + (zn.float() * w_zn.float()).sum()).backward()
        return [t.grad for t in leaves]

    for name, a, b in zip(("z", "attn", "mlp", "gate", "alpha", "beta"), run(True), run(False)):
        assert a.dtype == b.dtype, name
        assert rel_err(a, b) < TOL[dtype], name


def test_validation():
    _, d = make(2, 16, 64, torch.float32, seed=7)
    with pytest.raises(ValueError):
        ops.branch_lazy_update(d["z"], d["attn"][:, :8], d["mlp"], d["gate"], d["alpha"], d["beta"])
    with pytest.raises(ValueError):
        ops.branch_lazy_update(d["z"], d["attn"], d["mlp"], d["gate"][:1], d["alpha"], d["beta"])
    with pytest.raises(ValueError):
        ops.branch_lazy_update(d["z"], d["attn"].half(), d["mlp"], d["gate"], d["alpha"], d["beta"])
    with pytest.raises(ValueError):
        ops.branch_lazy_update(d["z"][..., :60], d["attn"][..., :60], d["mlp"][..., :60], d["gate"][:, :60],
                               d["alpha"][:60], d["beta"][:60])  # C not a multiple of 8


def test_unaligned_gate_view_and_empty_batch():
    """A gate view whose rows are not 16-byte aligned is copied before the call;
    an empty batch returns empty outputs and zero weight gradients."""
    _, d = make(2, 32, 64, torch.bfloat16, seed=9)
    t = torch.randn(2, 6 * 64 + 1, device="cuda").to(torch.bfloat16)
    gate = t[:, 1:65]  # starts 2 bytes into the row
    assert gate.data_ptr() % 16 != 0
    a = ops.branch_lazy_update(d["z"], d["attn"], d["mlp"], gate, d["alpha"], d["beta"])
    b = ops.branch_lazy_update(d["z"], d["attn"], d["mlp"], gate.contiguous(), d["alpha"], d["beta"])
    assert all(torch.equal(x, y) for x, y in zip(a, b))
    e = torch.empty(0, 16, 64, device="cuda", dtype=torch.bfloat16)
    ge = torch.empty(0, 64, device="cuda", dtype=torch.bfloat16)
    dz, zn = ops.branch_lazy_update(e, e, e, ge, d["alpha"], d["beta"])
    assert dz.shape == e.shape and zn.shape == e.shape
    g_attn, g_mlp, g_gate, ga, gb = ops.branch_lazy_update_bwd(None, e, e, e, ge, d["alpha"], d["beta"])
    assert g_gate.shape == (0, 64) and torch.count_nonzero(ga) == 0 and torch.count_nonzero(gb) == 0
