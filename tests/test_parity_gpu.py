"""Parity of the CUDA kernels (through the C ABI / operator layer) with the C oracle
and with the reference's golden vectors.

Forward ops and the per-cell gradients use the same fp32 fused-multiply-add
order as the oracle, so they are compared bit for bit; the exception is the
tensor-core materialisation backward (16-bit, L >= 2), whose grad_dz is held
to one unit in the last place.  Weight gradients are
reductions over cells (two-stage, fixed order on the GPU; fp64 in the oracle)
and are compared with a relative tolerance of 1e-5 of the largest magnitude.
Golden vectors from the reference's eager code: 1e-5 (fp32) / 2e-2 (bf16).
"""
from __future__ import annotations

import ctypes

import pytest
import torch

import flowmatching_lthc_b200 as F
from conftest import GOLDEN, close_16bit
from flowmatching_lthc_b200 import _lib, modules, ops, workloads
from oracle import lthc_oracle as O

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.bfloat16, torch.float16]
# (B, G, C): full slices, a ragged last slice (72 = 64 + 8), the minimum C, odd G,
# a single cell, the B/4 geometry
SHAPES = [(2, 4, 64), (1, 16, 72), (3, 3, 8), (2, 1, 128), (1, 16, 768)]
RTOL_REDUCTION = 1e-5
GOLD_TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2}


def same_bits(a: torch.Tensor, b: torch.Tensor) -> bool:
    a, b = a.detach().cpu(), b.detach().cpu()
    if a.shape != b.shape or a.dtype != b.dtype:
        return False
    iv = {4: torch.int32, 2: torch.int16}[a.element_size()]
    return torch.equal(a.contiguous().view(iv), b.contiguous().view(iv))


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.detach().cpu().double(), b.detach().cpu().double()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def rnd(*shape, dtype=torch.float32, std=1.0, mean=0.0, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * std + mean).to(dtype)


def device_status_ok() -> bool:
    st = ctypes.c_int(-1)
    _lib.call("lthc_device_status", ctypes.byref(st), torch.cuda.current_stream().cuda_stream)
    return st.value == 0


@pytest.fixture(autouse=True)
def _check_device_word():
    yield
    torch.cuda.synchronize()
    assert device_status_ok()


# ------------------------------------------------------------------ forward ops
@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("B,G,C", SHAPES)
@pytest.mark.parametrize("wdt", [torch.float32, torch.bfloat16])
def test_read_bit_exact(dt, B, G, C, wdt):
    x = rnd(B, 4 * G, 4 * G, C, dtype=dt, seed=1)
    a = torch.softmax(rnd(C, 16, seed=2), -1).to(wdt)
    z = F.read(x.cuda(), a.cuda())
    assert same_bits(z, O.read(x, a))


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("B,G,C", SHAPES)
def test_write_and_write_add_bit_exact(dt, B, G, C):
    x = rnd(B, 4 * G, 4 * G, C, dtype=dt, seed=3)
    dz = rnd(B, G * G, C, dtype=dt, seed=4)
    beta = rnd(C, 16, std=0.02, seed=5)
    assert same_bits(F.write(dz.cuda(), beta.cuda()), O.write(dz, beta))
    assert same_bits(F.write_add(x.cuda(), dz.cuda(), beta.cuda()), O.write_add(x, dz, beta))


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("L", [1, 3, 12])
@pytest.mark.parametrize("B,G,C", SHAPES[:4])
def test_materialise_bit_exact(dt, L, B, G, C):
    x0 = rnd(B, 4 * G, 4 * G, C, dtype=dt, seed=6)
    dz = [rnd(B, G * G, C, dtype=dt, std=0.1, seed=10 + l) for l in range(L)]
    beta = [rnd(C, 16, std=0.02, seed=40 + l) for l in range(L)]
    out = F.materialise(x0.cuda(), [d.cuda() for d in dz], [b.cuda() for b in beta])
    assert same_bits(out, O.materialise(x0, dz, beta))


def test_materialise_without_x0_and_in_place_write_add_via_abi():
    B, G, C, L = 2, 4, 64, 5
    dt = torch.bfloat16
    dz = [rnd(B, G * G, C, dtype=dt, seed=60 + l).cuda() for l in range(L)]
    beta = [rnd(C, 16, seed=70 + l).cuda() for l in range(L)]
    out = torch.empty(B, 4 * G, 4 * G, C, dtype=dt, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    _lib.call("lthc_materialise_fwd", None, _lib.ptr_array([d.data_ptr() for d in dz]),
              _lib.ptr_array([b.data_ptr() for b in beta]), 0, L, out.data_ptr(), B, G, C, 1, s)
    assert same_bits(out, O.materialise(None, [d.cpu() for d in dz], [b.cpu() for b in beta]))
    x = rnd(B, 4 * G, 4 * G, C, dtype=dt, seed=80).cuda()
    expect = O.write_add(x.cpu(), dz[0].cpu(), beta[0].cpu())
    _lib.call("lthc_write_add_fwd", x.data_ptr(), dz[0].data_ptr(), beta[0].data_ptr(), 0, x.data_ptr(), B, G, C, 1,
              s)
    assert same_bits(x, expect)


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("B,G,C", SHAPES[:4])
def test_lazy_update_bit_exact(dt, B, G, C):
    z = rnd(B, G * G, C, dtype=dt, seed=90)
    dz = rnd(B, G * G, C, dtype=dt, seed=91)
    a = torch.softmax(rnd(C, 16, seed=92), -1).to(dt)
    b = rnd(C, 16, std=0.02, mean=1.0, seed=93).to(dt)
    assert same_bits(F.lazy_update(z.cuda(), dz.cuda(), a.cuda(), b.cuda()), O.lazy_fwd(z, dz, a, b))


# ------------------------------------------------------------------ backward ops
@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("L", [1, 12])
@pytest.mark.parametrize("B,G,C", SHAPES)
def test_materialise_backward(dt, L, B, G, C):
    g = rnd(B, 4 * G, 4 * G, C, dtype=dt, seed=100)
    dz = [rnd(B, G * G, C, dtype=dt, std=0.1, seed=110 + l) for l in range(L)]
    beta = [rnd(C, 16, std=0.02, seed=130 + l) for l in range(L)]
    gdz, gb = ops.materialise_bwd(g.cuda(), [d.cuda() for d in dz], [b.cuda() for b in beta], True, True)
    rdz, rb = O.materialise_bwd(g, dz, beta)
    tc = ops.materialise_bwd_uses_tensor_cores(B, G, C, L, dt)
    for a_, b_ in zip(gdz, rdz):
        assert close_16bit(a_, b_) if tc else same_bits(a_, b_)
    assert rel_err(gb, rb) < RTOL_REDUCTION


# shapes the tensor-core backward takes: G = 8 (two stages per cell row pair), 16,
# 32 and 64 (half a cell row per stage); one and several 16-channel slices; the
# B/4 geometry with more tiles than SMs, so that CTAs straddle channel slices
TC_SHAPES = [(2, 8, 64, (2, 3, 12)), (1, 32, 32, (2, 12)), (1, 64, 16, (5,)), (3, 16, 48, (12,)),
             (8, 16, 768, (12,))]


@pytest.mark.parametrize("beta_f32", [True, False])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("B,G,C,L", [(b, g, c, l) for b, g, c, ls in TC_SHAPES for l in ls])
def test_materialise_backward_tensor_cores(beta_f32, dt, B, G, C, L):
    """grad_dz within one unit in the last place of the oracle's sequential fp32 sum,
    grad_beta within 1e-5; either gradient alone equals the fused call bit for bit
    and repeated calls are identical."""
    assert ops.materialise_bwd_uses_tensor_cores(B, G, C, L, dt)
    g = rnd(B, 4 * G, 4 * G, C, dtype=dt, seed=300 + L)
    dz = [rnd(B, G * G, C, dtype=dt, std=0.1, seed=310 + l) for l in range(L)]
    beta = [rnd(C, 16, std=0.02, seed=330 + l).to(torch.float32 if beta_f32 else dt) for l in range(L)]
    gc, dzc, bc = g.cuda(), [d.cuda() for d in dz], [b.cuda() for b in beta]
    gdz, gb = ops.materialise_bwd(gc, dzc, bc, True, True)
    rdz, rb = O.materialise_bwd(g, dz, beta)
    for l, (a_, b_) in enumerate(zip(gdz, rdz)):
        assert close_16bit(a_, b_), l
    assert rel_err(gb, rb) < RTOL_REDUCTION
    only_dz, _ = ops.materialise_bwd(gc, dzc, bc, True, False)
    _, only_b = ops.materialise_bwd(gc, dzc, bc, False, True)
    assert all(same_bits(a_, b_) for a_, b_ in zip(only_dz, gdz))
    assert same_bits(only_b, gb)
    again, gb_again = ops.materialise_bwd(gc, dzc, bc, True, True)
    assert all(same_bits(a_, b_) for a_, b_ in zip(again, gdz)) and same_bits(gb_again, gb)


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("B,G,C", SHAPES[:4])
def test_read_backward(dt, B, G, C):
    x = rnd(B, 4 * G, 4 * G, C, dtype=dt, seed=150)
    gz = rnd(B, G * G, C, dtype=dt, seed=151)
    a = torch.softmax(rnd(C, 16, seed=152), -1)
    gx, ga = ops.read_bwd(x.cuda(), gz.cuda(), a.cuda(), True, True)
    assert same_bits(gx, O.write(gz, a))
    assert rel_err(ga, O.weight_grad(x, [gz])[0]) < RTOL_REDUCTION
    # accumulating onto a gradient X already holds (the patch embedding's backward
    # passes the materialisation's gradient): base + alpha (.) bcast(grad_z), one rounding
    base = rnd(B, 4 * G, 4 * G, C, dtype=dt, seed=153)
    gx2, ga2 = ops.read_bwd(x.cuda(), gz.cuda(), a.cuda(), True, True, base.cuda())
    assert same_bits(gx2, O.write_add(base, gz, a))
    assert torch.equal(ga2, ga)
    # both gradients come from one fused pass; either alone from the write / weight-gradient kernels
    gx_only, _ = ops.read_bwd(x.cuda(), gz.cuda(), a.cuda(), True, False)
    _, ga_only = ops.read_bwd(x.cuda(), gz.cuda(), a.cuda(), False, True)
    assert same_bits(gx_only, gx)
    assert rel_err(ga_only, ga) < RTOL_REDUCTION


@pytest.mark.parametrize("dt", DTYPES)
@pytest.mark.parametrize("B,G,C", SHAPES[:4])
def test_lazy_backward(dt, B, G, C):
    gzo = rnd(B, G * G, C, dtype=dt, seed=160)
    dz = rnd(B, G * G, C, dtype=dt, seed=161)
    a = torch.softmax(rnd(C, 16, seed=162), -1).to(dt)
    b = rnd(C, 16, std=0.02, mean=1.0, seed=163).to(dt)
    gdz, ga, gb = ops.lazy_update_bwd(gzo.cuda(), dz.cuda(), a.cuda(), b.cuda())
    rdz, ra, rb = O.lazy_bwd(gzo, dz, a, b)
    assert same_bits(gdz, rdz)
    assert rel_err(ga, ra) < RTOL_REDUCTION and rel_err(gb, rb) < RTOL_REDUCTION


def test_weight_grad_is_deterministic():
    B, G, C, L = 4, 16, 128, 12
    g = rnd(B, 4 * G, 4 * G, C, dtype=torch.bfloat16, seed=170).cuda()
    dz = [rnd(B, G * G, C, dtype=torch.bfloat16, seed=171 + l).cuda() for l in range(L)]
    first = F.weight_grad(g, dz)
    for _ in range(3):
        assert same_bits(F.weight_grad(g, dz), first)


# --------------------------------------------------------- autograd composition
def _torch_reference(x0, dzs, read_logits, write_weights):
    """The reference's eager formulas (local_thc.py:1204-1223, 1261-1283, 1325-1328,
    1368-1372) in fp64 autograd."""
    B, H, _, C = x0.shape
    G = H // 4
    alpha = torch.softmax(read_logits, -1)

    def read(x):
        xv = x.view(B, G, 4, G, 4, C)
        a = alpha.view(C, 4, 4).permute(1, 2, 0)
        return (xv * a[None, None, :, None, :, :]).sum(dim=(2, 4)).reshape(B, G * G, C)

    def write(dz, w):
        b = w.view(C, 4, 4).permute(1, 2, 0)
        return (dz.view(B, G, G, C)[:, :, None, :, None, :] * b[None, None, :, None, :, :]).reshape(B, H, H, C)

    z = read(x0)
    zs = [z]
    for d, w in zip(dzs, write_weights):
        z = z + (alpha * w).sum(-1) * d
        zs.append(z)
    xl = x0
    for d, w in zip(dzs, write_weights):
        xl = xl + write(d, w)
    return zs[-1], xl


def test_autograd_through_the_lthc_interface_matches_eager_fp64():
    torch.manual_seed(0)
    B, G, C, L = 2, 4, 64, 12
    x0 = torch.randn(B, 4 * G, 4 * G, C, device="cuda")
    dzs = [torch.randn(B, G * G, C, device="cuda") * 0.1 for _ in range(L)]
    read = modules.SharedLocalRead(4 * G, G, C, C).cuda()
    writes = [modules.LayerLocalWrite(4 * G, G, C, C).cuda() for _ in range(L)]
    with torch.no_grad():
        read.read_logits.normal_()
        for w in writes:
            w.write_weight.normal_(1.0, 0.05)
    gz_up = torch.randn(B, G * G, C, device="cuda")
    gx_up = torch.randn(B, 4 * G, 4 * G, C, device="cuda")

    x0a = x0.clone().requires_grad_(True)
    dza = [d.clone().requires_grad_(True) for d in dzs]
    z = read.read(x0a)
    for d, w in zip(dza, writes):
        z = modules.lazy_workspace_update(z, d, read, w)
    xl = modules.final_accumulate(x0a, dza, writes)
    params = [read.read_logits] + [w.write_weight for w in writes]
    ours = torch.autograd.grad((z * gz_up).sum() + (xl * gx_up).sum(), [x0a, *dza, *params])

    x0d = x0.double().requires_grad_(True)
    dzd = [d.double().requires_grad_(True) for d in dzs]
    pd = [p.detach().double().requires_grad_(True) for p in params]
    zr, xr = _torch_reference(x0d, dzd, pd[0], pd[1:])
    assert rel_err(z, zr) < 1e-5 and rel_err(xl, xr) < 1e-5
    theirs = torch.autograd.grad((zr * gz_up.double()).sum() + (xr * gx_up.double()).sum(), [x0d, *dzd, *pd])
    for a_, b_ in zip(ours, theirs):
        assert rel_err(a_, b_) < 1e-5


# ------------------------------------------------------------------ golden vectors
@pytest.mark.parametrize("name", ["g4_c40_f32", "g4_c40_bf16", "g16_c8_f32", "g2_c64_bf16"])
def test_golden_vectors_through_cuda(name):
    d = torch.load(GOLDEN / f"{name}.pt")
    dt = d["x"].dtype
    tol = GOLD_TOL[dt]
    cu = {k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in d.items()}
    a = cu["R"].to(dt)
    assert rel_err(F.read(cu["x"], a), d["read_z"]) < tol
    assert rel_err(F.write(cu["dz"][0], cu["P"][0].to(dt)), d["write_out"]) < tol
    assert rel_err(F.write_add(cu["x"], cu["dz"][0], cu["P"][0].to(dt)), d["write_add_out"]) < tol
    assert rel_err(F.lazy_update(cu["read_z"], cu["dz"][0], a, cu["P"][0].to(dt)), d["lazy_z"]) < tol
    P = list(cu["P"])
    assert rel_err(F.materialise(cu["x"], list(cu["dz_small"]), P), d["mat_out"]) < tol
    gdz, gP = ops.materialise_bwd(cu["g_x"], list(cu["dz_small"]), P, True, True)
    assert rel_err(torch.stack(gdz), d["mat_gdz"]) < tol
    assert rel_err(gP, d["mat_gP"]) < tol
    gx, gR = ops.read_bwd(cu["x"], cu["g_z"], a, True, True)
    assert rel_err(gx, d["read_gx"]) < tol and rel_err(gR, d["read_gR"]) < tol


# ------------------------------------------------------------- full-size properties
@pytest.mark.slow
def test_materialise_config2_full_size():
    """BASELINE config 2 (B=64, bf16): sampled batch elements of the forward bit-exact
    against the oracle (cells are independent) and of the tensor-core backward's
    grad_dz within one unit in the last place, the fp32 weight gradient of the
    full batch against the oracle, and run-to-run determinism."""
    cfg = workloads.config2(B=64, device="cuda", seed=0)
    x0, dz, P = cfg["x0"], cfg["dz"], cfg["P"]
    out = F.materialise(x0, dz, P)
    for b in (0, 37, 63):
        ref = O.materialise(x0[b:b + 1].cpu(), [d[b:b + 1].cpu() for d in dz], [p.cpu() for p in P])
        assert same_bits(out[b:b + 1], ref)
    assert same_bits(F.materialise(x0, dz, P), out)
    g = workloads.residual(64, 16, 768, seed=5, device="cuda", dtype=torch.bfloat16)
    gdz, gb = ops.materialise_bwd(g, dz, P, True, True)
    assert ops.materialise_bwd_uses_tensor_cores(64, 16, 768, 12, torch.bfloat16)
    for b in (1, 62):
        rdz, _ = O.materialise_bwd(g[b:b + 1].cpu(), [d[b:b + 1].cpu() for d in dz], [p.cpu() for p in P])
        for l in range(12):
            assert close_16bit(gdz[l][b:b + 1], rdz[l])
    rb = O.weight_grad(g.cpu(), [d.cpu() for d in dz])
    assert rel_err(gb, rb) < RTOL_REDUCTION
    _, gb2 = ops.materialise_bwd(g, dz, P, False, True)
    assert same_bits(gb2, gb)


@pytest.mark.slow
def test_materialise_and_read_beyond_2pow31_elements():
    """B = 700 at the B/4 shape: the residual has 2.2e9 elements, more than a 32-bit
    offset can address (the reference's Triton materialisation wraps there).  The
    first and last images must match the oracle bit for bit."""
    B = 700
    cfg = workloads.config2(B=B, device="cuda", seed=9)
    x0, dz, P = cfg["x0"], cfg["dz"], cfg["P"]
    assert x0.numel() > 2**31
    out = F.materialise(x0, dz, P)
    alpha = torch.softmax(cfg["R"], -1)
    z = F.read(out, alpha)
    for b in (0, B - 1):
        ref = O.materialise(x0[b:b + 1].cpu(), [d[b:b + 1].cpu() for d in dz], [p.cpu() for p in P])
        assert same_bits(out[b:b + 1], ref)
        assert same_bits(z[b:b + 1], O.read(ref, alpha.cpu()))


@pytest.mark.slow
def test_lazy_identity_full_size_fp32():
    """read(X_0 + sum_l P_l dZ_l) == read(X_0) + sum_l Gamma_l dZ_l at the B/4 geometry."""
    cfg = workloads.config2(B=8, device="cuda", seed=1, dtype=torch.float32)
    alpha = torch.softmax(torch.randn(768, 16, device="cuda"), -1)
    z = F.read(cfg["x0"], alpha)
    for d, p in zip(cfg["dz"], cfg["P"]):
        z = F.lazy_update(z, d, alpha, p)
    naive = F.read(F.materialise(cfg["x0"], cfg["dz"], cfg["P"]), alpha)
    assert rel_err(z, naive) < 1e-5


# ------------------------------------------------------------------ error paths
def test_validation_on_device_pointers():
    x = torch.zeros(1, 16, 16, 64, dtype=torch.bfloat16, device="cuda")
    z = torch.zeros(1, 16, 64, dtype=torch.bfloat16, device="cuda")
    a = torch.zeros(64, 16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    with pytest.raises(_lib.LthcError) as ei:
        _lib.call("lthc_read_fwd", x.data_ptr() + 2, a.data_ptr(), 0, z.data_ptr(), 1, 4, 64, 1, s)
    assert ei.value.status == 4
    gw = torch.zeros(1, 64, 16, device="cuda")
    ws = torch.zeros(16, dtype=torch.uint8, device="cuda")
    with pytest.raises(_lib.LthcError) as ei:
        _lib.call("lthc_weight_grad", x.data_ptr(), _lib.ptr_array([z.data_ptr()]), 1, gw.data_ptr(), ws.data_ptr(),
                  16, 1, 4, 64, 1, s)
    assert ei.value.status == 5
    with pytest.raises(ValueError):
        F.read(x, torch.zeros(32, 16, device="cuda"))


def test_empty_batch_on_device():
    x = torch.zeros(0, 64, 64, 64, device="cuda", dtype=torch.bfloat16)
    a = torch.zeros(64, 16, device="cuda")
    assert F.read(x, a).shape == (0, 256, 64)
    gw = F.weight_grad(x, [torch.zeros(0, 256, 64, device="cuda", dtype=torch.bfloat16)])
    assert gw.shape == (1, 64, 16) and int(torch.count_nonzero(gw)) == 0


# -------------------------------------------------------------- graph capture
def test_cuda_graph_capture_replay():
    B, G, C, L = 2, 16, 128, 12
    x0 = rnd(B, 4 * G, 4 * G, C, dtype=torch.bfloat16, seed=200).cuda()
    dz = [rnd(B, G * G, C, dtype=torch.bfloat16, seed=201 + l).cuda() for l in range(L)]
    P = [rnd(C, 16, std=0.02, seed=220 + l).cuda() for l in range(L)]
    expect = F.materialise(x0, dz, P)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        F.materialise(x0, dz, P)  # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = F.materialise(x0, dz, P)
    g.replay()
    torch.cuda.synchronize()
    assert same_bits(out, expect)


# ------------------------------------------------------------------ failure detection
def test_bounded_wait_gives_up_and_context_stays_usable():
    """A wait on a barrier nothing completes gives up after its limit, the device
    error word reports LTHC_ERR_TIMEOUT, and the next kernels run normally."""
    res = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    _lib.call("lthc_selftest_wait_timeout", 50, res.data_ptr(), s)
    st = ctypes.c_int(-1)
    _lib.call("lthc_device_status", ctypes.byref(st), s)
    assert st.value == 8 and int(res.item()) == 1
    assert device_status_ok()  # reading cleared the word
    B, G, C = 1, 4, 64
    x0 = rnd(B, 4 * G, 4 * G, C, dtype=torch.bfloat16, seed=300)
    dz = [rnd(B, G * G, C, dtype=torch.bfloat16, seed=301)]
    beta = [rnd(C, 16, seed=302)]
    out = F.materialise(x0.cuda(), [d.cuda() for d in dz], [b.cuda() for b in beta])
    assert same_bits(out, O.materialise(x0, dz, beta))


def test_materialise_from_host_buffers_pipelined():
    """Chunked, stream-overlapped materialisation from pinned host buffers gives the
    same bits as the device call (batch not a multiple of the chunk)."""
    from flowmatching_lthc_b200.host import HostMaterialiser

    B, G, C, L = 11, 4, 64, 12
    x0 = rnd(B, 4 * G, 4 * G, C, dtype=torch.bfloat16, seed=400)
    dz = [rnd(B, G * G, C, dtype=torch.bfloat16, std=0.1, seed=401 + l) for l in range(L)]
    P = [rnd(C, 16, std=0.02, seed=420 + l).cuda() for l in range(L)]
    hm = HostMaterialiser(chunk=4, depth=2)
    out = torch.empty_like(x0).pin_memory()
    for _ in range(2):  # second call reuses the staging ring
        out.zero_()
        hm(x0.pin_memory(), [d.pin_memory() for d in dz], P, out)
        torch.cuda.synchronize()
        assert same_bits(out, O.materialise(x0, dz, [p.cpu() for p in P]))


def test_torch_compile_fullgraph_forward_and_backward():
    """The ops trace under torch.compile (fake implementations + registered autograd)
    and the compiled graph gives the eager results bit for bit (weight gradients summed over
    several uses: up to fp32 reassociation)."""
    torch._dynamo.reset()
    B, G, C, L = 2, 4, 64, 3
    dt = torch.bfloat16
    x0 = rnd(B, 4 * G, 4 * G, C, dtype=dt, seed=500).cuda()
    dz = [rnd(B, G * G, C, dtype=dt, std=0.1, seed=501 + l).cuda() for l in range(L)]
    P = [rnd(C, 16, std=0.02, mean=1.0, seed=510 + l).cuda() for l in range(L)]
    # alpha enters as an fp32 leaf: a softmax or bf16 cast inside the graph would be
    # fused by the compiler with its own rounding, which is not what this test checks.
    alpha0 = torch.softmax(rnd(C, 16, seed=520), -1).cuda()

    def f(x0, dz, P, alpha):
        z = ops.read(x0, alpha)
        for d, p in zip(dz, P):
            z = ops.lazy_update(z, d, alpha, p)
        xl = ops.materialise(x0, dz, P)
        return (z.float().square().sum() + xl.float().square().sum()), z, xl

    def run(fn):
        a = [x0.clone().requires_grad_(True)] + [d.clone().requires_grad_(True) for d in dz]
        ps = [p.clone().requires_grad_(True) for p in P]
        lg = alpha0.clone().requires_grad_(True)
        loss, z, xl = fn(a[0], a[1:], ps, lg)
        loss.backward()
        return [z, xl] + [t.grad for t in a + ps + [lg]]

    eager = run(f)
    compiled = run(torch.compile(f, fullgraph=True))
    for e, c in zip(eager, compiled):
        assert same_bits(c, e) or rel_err(c, e) < RTOL_REDUCTION


def test_direct_call_path_matches_the_operator():
    """ops.call: the direct CUDA path (no autograd needed) gives the operator's
    bits; with an input that requires grad it goes through the operator and
    records the autograd graph."""
    x = rnd(2, 16, 16, 64, dtype=torch.bfloat16, seed=600).cuda()
    alpha = rnd(64, 16, dtype=torch.bfloat16, seed=601).cuda()
    ref = ops.read(x, alpha)
    assert same_bits(ops.call(ops.read, x, alpha), ref)
    xr = x.clone().requires_grad_(True)
    out = ops.call(ops.read, xr, alpha)
    assert out.grad_fn is not None and same_bits(out, ref)
    with torch.no_grad():
        out2 = ops.call(ops.read, xr, alpha)
    assert out2.grad_fn is None and same_bits(out2, ref)
