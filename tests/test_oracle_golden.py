"""Pins the C oracle against golden vectors produced by the reference's own eager
PyTorch code (tests/golden/make_golden.py) and against the algebraic identities
the reference documents.  CPU only."""
from __future__ import annotations

import pytest
import torch

from conftest import GOLDEN
from oracle import lthc_oracle as O

CASES = ["g4_c40_f32", "g4_c40_bf16", "g16_c8_f32", "g2_c64_bf16"]
# fp32: 1e-5 relative; bf16: 2e-2 (the reference's eager bf16 path rounds after
# every product/sum, the oracle once)
TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2}


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double(), b.double()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


@pytest.fixture(scope="module", params=CASES)
def case(request):
    return torch.load(GOLDEN / f"{request.param}.pt")


def test_read(case):
    dt = case["x"].dtype
    assert rel_err(O.read(case["x"], case["R"].to(dt)), case["read_z"]) < TOL[dt]


def test_read_backward(case):
    dt = case["x"].dtype
    # grad_x = alpha (.) grad_z broadcast over the cell == write(grad_z, alpha)
    assert rel_err(O.write(case["g_z"], case["R"].to(dt)), case["read_gx"]) < TOL[dt]
    assert rel_err(O.weight_grad(case["x"], [case["g_z"]])[0], case["read_gR"]) < TOL[dt]


def test_write_and_write_add(case):
    dt = case["x"].dtype
    P0 = case["P"][0].to(dt)
    assert rel_err(O.write(case["dz"][0], P0), case["write_out"]) < TOL[dt]
    assert rel_err(O.write_add(case["x"], case["dz"][0], P0), case["write_add_out"]) < TOL[dt]


def test_write_backward(case):
    dt = case["x"].dtype
    gdz, gP = O.materialise_bwd(case["g_x"], [case["dz"][0]], [case["P"][0].to(dt)])
    assert rel_err(gdz[0], case["write_gdz"]) < TOL[dt]
    assert rel_err(gP[0], case["write_gP"]) < TOL[dt]
    assert rel_err(gdz[0], case["write_add_gdz"]) < TOL[dt]
    assert torch.equal(case["write_add_gx"], case["g_x"])  # identity branch of write_add


def test_gamma_and_lazy(case):
    dt = case["x"].dtype
    a, p0 = case["R"].to(dt), case["P"][0].to(dt)
    assert rel_err(O.lazy_fwd(case["read_z"], case["dz"][0], a, p0), case["lazy_z"]) < TOL[dt]
    gdz, ga, gb = O.lazy_bwd(case["g_z"], case["dz"][0], a, p0)
    assert rel_err(gdz, case["lazy_gdz"]) < TOL[dt]
    assert rel_err(ga, case["lazy_gR"]) < TOL[dt]
    assert rel_err(gb, case["lazy_gP"]) < TOL[dt]
    assert torch.equal(case["lazy_gz"], case["g_z"])  # identity branch of the recurrence


def test_materialise(case):
    dt = case["x"].dtype
    P = list(case["P"])
    out = O.materialise(case["x"], list(case["dz_small"]), P)
    assert rel_err(out, case["mat_out"]) < TOL[dt]


def test_materialise_backward(case):
    dt = case["x"].dtype
    P = list(case["P"])
    gdz, gP = O.materialise_bwd(case["g_x"], list(case["dz_small"]), P)
    assert rel_err(torch.stack(gdz), case["mat_gdz"]) < TOL[dt]
    assert rel_err(gP, case["mat_gP"]) < TOL[dt]
    assert torch.equal(case["mat_gx0"], case["g_x"])  # grad X_0 is grad X_L


def test_lazy_identity_read_of_write_is_gamma():
    """R(P_l(dZ)) = Gamma_l (.) dZ (the identity behind the lazy recurrence,
    docs/kernel_note.md:49-53 of the reference)."""
    torch.manual_seed(0)
    C, G = 24, 3
    alpha = torch.softmax(torch.randn(C, 16), -1)
    beta = torch.randn(C, 16) * 0.02 + 1.0
    dz = torch.randn(2, G * G, C)
    lhs = O.read(O.write(dz, beta), alpha)
    gamma = (alpha * beta).sum(-1)
    assert rel_err(lhs, gamma * dz) < 1e-6


def test_lazy_equals_naive_recurrence():
    """Z after L lazy updates equals the read of the materialised residual (fp64-exact
    algebra, fp32 arithmetic): read(X_0 + sum_l P_l dZ_l) == read(X_0) + sum_l Gamma_l dZ_l."""
    torch.manual_seed(1)
    C, G, L = 16, 2, 5
    alpha = torch.softmax(torch.randn(C, 16), -1)
    betas = [torch.randn(C, 16) * 0.05 + 1.0 for _ in range(L)]
    x0 = torch.randn(3, 4 * G, 4 * G, C)
    dzs = [torch.randn(3, G * G, C) for _ in range(L)]
    z = O.read(x0, alpha)
    for d, b in zip(dzs, betas):
        z = O.lazy_fwd(z, d, alpha, b)
    naive = O.read(O.materialise(x0, dzs, betas), alpha)
    assert rel_err(z, naive) < 1e-5


def test_materialise_is_sequential_write_add_fp32():
    torch.manual_seed(2)
    C, G, L = 8, 2, 12
    betas = [torch.randn(C, 16) for _ in range(L)]
    x = torch.randn(2, 4 * G, 4 * G, C)
    dzs = [torch.randn(2, G * G, C) for _ in range(L)]
    seq = x
    for d, b in zip(dzs, betas):
        seq = O.write_add(seq, d, b)
    assert rel_err(O.materialise(x, dzs, betas), seq) < 1e-6


def test_empty_batch():
    C, G = 8, 2
    x = torch.empty(0, 4 * G, 4 * G, C)
    assert O.read(x, torch.ones(C, 16)).shape == (0, G * G, C)
    gw = O.weight_grad(x, [torch.empty(0, G * G, C)])
    assert gw.shape == (1, C, 16) and torch.count_nonzero(gw) == 0


def test_output_rounding_matches_torch_casts():
    """The oracle rounds fp32 results to fp16/bf16 with IEEE round-to-nearest-even,
    like torch's casts (values spanning subnormals to overflow)."""
    from flowmatching_lthc_b200.workloads import cell_major_to_nhwc

    torch.manual_seed(3)
    C, G = 8, 8
    scale = torch.logspace(-9, 5, G * G).view(1, G * G, 1)
    for dt in (torch.float16, torch.bfloat16):
        dz = (torch.randn(1, G * G, C) * scale).to(dt)
        beta = torch.rand(C, 16) * 3
        out = O.write(dz, beta)
        ref = cell_major_to_nhwc(dz.float()[:, :, None, :] * beta.t()[None, None]).to(dt)
        assert torch.equal(out.float(), ref.float())


# ---- final-layer prologue (FinalLayerSharedAdaLN: RMSNorm + modulate) ----------
FINAL_CASES = ["final_t64_c768_bf16", "final_t16_c40_f32", "final_t8_c1024_bf16"]


def exact_fraction(a: torch.Tensor, b: torch.Tensor) -> float:
    return (a == b).float().mean().item()


@pytest.fixture(scope="module", params=FINAL_CASES)
def final_case(request):
    return torch.load(GOLDEN / f"{request.param}.pt")


def test_final_norm_modulate_forward(final_case):
    """Op-by-op rounding as the reference: the outputs agree exactly except where
    the mean of squares, summed in another order, moves an element across a
    rounding boundary of the activation dtype (16-bit); fp32 within 1e-5."""
    c = final_case
    C = c["meta"]["C"]
    shift, scale = c["t2"][:, :C], c["t2"][:, C:]
    m = O.final_fwd(c["x"], c["norm_weight"], shift, scale, c["meta"]["eps"])
    assert m.dtype == c["m"].dtype
    if m.dtype != torch.float32:  # fp32 has no output rounding to absorb the reduction order
        assert exact_fraction(m, c["m"]) > 0.999
    assert rel_err(m, c["m"]) < TOL[c["x"].dtype]
    if "layer_out" in c:  # fp32: the full layer = Linear(m)
        out = torch.nn.functional.linear(m, c["linear_weight"], c["linear_bias"])
        assert rel_err(out, c["layer_out"]) < 1e-5


def test_final_norm_modulate_backward(final_case):
    c = final_case
    C = c["meta"]["C"]
    dt = c["x"].dtype
    gx, gw, gsh, gsc = O.final_bwd(c["g_m"], c["x"], c["norm_weight"], c["t2"][:, C:], c["meta"]["eps"])
    if dt != torch.float32:
        assert exact_fraction(gx, c["gx"]) > 0.99
    assert rel_err(gx, c["gx"]) < TOL[dt]
    assert rel_err(gw, c["g_norm_weight"]) < 1e-5
    # shift / scale gradients are sums over tokens, rounded once to the parameter dtype
    assert rel_err(gsh.to(dt), c["g_shift"]) < TOL[dt]
    assert rel_err(gsc.to(dt), c["g_scale"]) < TOL[dt]


# ---- branch epilogue fused with the lazy update --------------------------------
# (WorkspaceSharedAdaLNBranch.forward's output sum, then lazy_workspace_update)
BRANCH_CASES = ["branch_g4_c768_bf16", "branch_g4_c40_f32", "branch_g4_c64_f16"]
BRANCH_TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 5e-3}


@pytest.fixture(scope="module", params=BRANCH_CASES)
def branch_case(request):
    return torch.load(GOLDEN / f"{request.param}.pt")


def test_branch_lazy_forward(branch_case):
    """dz is the reference's op-by-op sum bit for bit (one rounding per op, as
    torch rounds); z' differs from the reference's z + gamma*dz only by gamma kept
    in fp32 and one rounding of the fused multiply-add."""
    c = branch_case
    dt = c["z"].dtype
    dz, zn = O.branch_fwd(c["z"], c["dz_attn"], c["mlp_out"], c["gate"], c["R"].to(dt), c["P"].to(dt))
    assert torch.equal(dz, c["dz"])
    assert rel_err(zn, c["z_next"]) < BRANCH_TOL[dt]
    assert exact_fraction(zn, c["z_next"]) > 0.98
    # the same as the unfused lazy update applied to that dz
    assert torch.equal(zn, O.lazy_fwd(c["z"], dz, c["R"].to(dt), c["P"].to(dt)))


@pytest.mark.parametrize("tag", ["both", "lazy_only"])
def test_branch_lazy_backward(branch_case, tag):
    c = branch_case
    dt = c["z"].dtype
    tol = BRANCH_TOL[dt]
    g_dz = c["g_dz"] if tag == "both" else None
    g_attn, g_mlp, g_gate, ga, gb = O.branch_bwd(g_dz, c["g_zn"], c["dz"], c["mlp_out"], c["gate"], c["R"].to(dt),
                                                 c["P"].to(dt))
    assert rel_err(g_attn, c[f"{tag}_gattn"]) < tol
    assert rel_err(g_mlp, c[f"{tag}_gmlp"]) < tol
    assert rel_err(g_gate.to(dt), c[f"{tag}_ggate"]) < tol
    assert rel_err(ga, c[f"{tag}_gR"]) < tol
    assert rel_err(gb, c[f"{tag}_gP"]) < tol
    assert torch.equal(c[f"{tag}_gz"], c["g_zn"])  # identity branch of the recurrence
    if tag == "both":  # gamma's rounding only enters through gamma * g_zn, small beside g_dz
        assert exact_fraction(g_attn, c[f"{tag}_gattn"]) > 0.98


def test_branch_lazy_empty_and_single_row():
    for b, t in ((0, 16), (2, 0), (1, 1)):
        z = torch.randn(b, t, 16)
        gate = torch.randn(b, 16)
        a, p = torch.rand(16, 16), torch.randn(16, 16)
        dz, zn = O.branch_fwd(z, z * 0.5, z * 2, gate, a, p)
        assert dz.shape == z.shape and zn.shape == z.shape
        g_attn, g_mlp, g_gate, ga, gb = O.branch_bwd(None, z, dz, z, gate, a, p)
        assert g_gate.shape == (b, 16)
        if b * t == 0:
            assert torch.count_nonzero(ga) == 0 and torch.count_nonzero(g_gate) == 0
