"""PyTorch operators over the C-ABI CUDA library.

Each operator is a ``torch.library.custom_op`` in the ``lthc_b200`` namespace with
a CUDA implementation (a call into ``liblthc_b200.so`` on the current stream), a
fake implementation for ``torch.compile`` tracing and an autograd formula whose
backward is itself a custom op.  Outputs and scratch come from the PyTorch
caching allocator; the library never allocates.  Only CUDA tensors are
accepted: there is no CPU implementation and no fallback.

The bottom of the file mirrors the reference's ``jit_thc::`` Triton op surface
(``flowmatching_lthc/models/local_thc_triton_kernels.py``) with the same names,
argument order and legacy read/write naming, so code written against those ops
can switch by changing its import.
"""
from __future__ import annotations

import contextlib
import ctypes
import math
from typing import Sequence

import torch
from torch import Tensor

from torch._subclasses.fake_tensor import FakeTensor
from torch.utils._python_dispatch import _get_current_dispatch_mode as _current_dispatch_mode

from . import _lib

_DTYPE_CODE = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16}
MAX_LAYERS = 12


# ---------------------------------------------------------------------------
# validation helpers (ValueError, as the reference ops raise on bad shapes,
# e.g. local_thc_triton_kernels.py:1387-1390)
# ---------------------------------------------------------------------------
def _code(t: Tensor, what: str) -> int:
    try:
        return _DTYPE_CODE[t.dtype]
    except KeyError:
        raise ValueError(f"{what}: unsupported dtype {t.dtype} (float32, bfloat16 or float16)") from None


def _require_cuda(*ts: Tensor) -> None:
    for t in ts:
        if t.device.type != "cuda":
            raise ValueError(f"LTHC ops run on CUDA tensors only (got a {t.device} tensor); there is no CPU path")


def _hi_geom(x: Tensor, what: str) -> tuple[int, int, int]:
    if x.dim() != 4:
        raise ValueError(f"{what}: expected NHWC [B,H,W,C], got {tuple(x.shape)}")
    b, h, w, c = x.shape
    if h != w or h % 4 != 0:
        raise ValueError(f"{what}: expected a square residual grid divisible by 4, got {tuple(x.shape)}")
    _check_channels(c, what)
    return b, h // 4, c


def _lo_geom(z: Tensor, what: str) -> tuple[int, int, int]:
    if z.dim() != 3:
        raise ValueError(f"{what}: expected workspace [B,N,C], got {tuple(z.shape)}")
    b, n, c = z.shape
    g = math.isqrt(n)
    if g * g != n or g == 0:
        raise ValueError(f"{what}: workspace token count {n} is not a non-zero square")
    _check_channels(c, what)
    return b, g, c


def _check_channels(c: int, what: str) -> None:
    if c % 8 != 0 or c < 8:
        raise ValueError(f"{what}: channel count {c} must be a positive multiple of 8")


def _check_weight(w: Tensor, c: int, what: str) -> None:
    if tuple(w.shape) != (c, 16):
        raise ValueError(f"{what}: expected weight [{c},16], got {tuple(w.shape)}")


def _guard(t: Tensor):
    """Make t's GPU current for the C call (the library launches on the current
    device); a no-op context when it already is."""
    idx = t.device.index
    if idx is None or torch.cuda.current_device() == idx:
        return contextlib.nullcontext()
    return torch.cuda.device(idx)


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(t: Tensor) -> int:
    """The current CUDA stream of t's device as a raw handle (without building a
    torch.cuda.Stream object when torch offers the raw query)."""
    if _raw_stream is not None:
        return _raw_stream(t.device.index if t.device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(t.device).cuda_stream


# The CUDA implementation of each operator, for calls that need neither autograd
# nor a tracer (see call()).
_DIRECT: dict = {}


def _custom_op(name: str):
    """torch.library.custom_op in the lthc_b200 namespace, CUDA only; the undecorated
    implementation is kept for the direct call path."""
    def deco(fn):
        op = torch.library.custom_op(f"lthc_b200::{name}", mutates_args=(), device_types="cuda")(fn)
        _DIRECT[id(op)] = fn
        return op
    return deco


def _tensors(args):
    for a in args:
        if isinstance(a, Tensor):
            yield a
        elif isinstance(a, (list, tuple)):
            yield from (t for t in a if isinstance(t, Tensor))


def call(op, *args):
    """Run `op` on args.  Calls that need no autograd graph (grad disabled or no
    input requiring grad), are not being traced and hold real CUDA tensors go
    straight to the CUDA implementation and skip the dispatcher's per-call cost
    (tens of microseconds, comparable to the kernels of a small batch); every
    other call goes through the registered operator."""
    ts = list(_tensors(args))
    fn = _DIRECT.get(id(op))
    if (fn is None or torch.compiler.is_compiling() or _current_dispatch_mode() is not None
            or any(t.device.type != "cuda" or isinstance(t, FakeTensor) for t in ts)
            or (torch.is_grad_enabled() and any(t.requires_grad for t in ts))):
        return op(*args)
    return fn(*args)


def _workspace(nbytes: int, device: torch.device) -> Tensor:
    # 16-byte aligned (the caching allocator returns 512-byte aligned blocks)
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)


def _p(t: Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# ---------------------------------------------------------------------------
# read: residual [B,4G,4G,C] -> workspace [B,G*G,C]
# ---------------------------------------------------------------------------
@_custom_op("read")
def read(x: Tensor, alpha: Tensor) -> Tensor:
    """z[b,cell,c] = sum_r alpha[c,r] x[b,cell,r,c]  (SharedLocalRead.read, local_thc.py:1211-1223)."""
    _require_cuda(x, alpha)
    b, g, c = _hi_geom(x, "read")
    _check_weight(alpha, c, "read")
    x, alpha = x.contiguous(), alpha.contiguous()
    z = torch.empty((b, g * g, c), device=x.device, dtype=x.dtype)
    with _guard(x):
        _lib.call("lthc_read_fwd", x.data_ptr(), alpha.data_ptr(), _code(alpha, "read"), z.data_ptr(), b, g, c,
                  _code(x, "read"), _stream(x))
    return z


@read.register_fake
def _(x: Tensor, alpha: Tensor) -> Tensor:
    b, h, _, c = x.shape
    return x.new_empty((b, (h // 4) * (h // 4), c))


@_custom_op("read_bwd")
def read_bwd(x: Tensor, grad_z: Tensor, alpha: Tensor, need_grad_x: bool, need_grad_alpha: bool,
             grad_x_in: Tensor | None = None) -> tuple[Tensor, Tensor]:
    """grad_x = (grad_x_in +) alpha (.) grad_z broadcast, fp32 accumulation and one
    rounding; grad_alpha = sum x*grad_z (fp32 [C,16])."""
    _require_cuda(x, grad_z, alpha)
    b, g, c = _hi_geom(x, "read_bwd")
    x, grad_z, alpha = x.contiguous(), grad_z.contiguous(), alpha.contiguous()
    if grad_x_in is not None:
        _require_cuda(grad_x_in)
        if grad_x_in.shape != x.shape:
            raise ValueError(f"read_bwd: grad_x_in must be {tuple(x.shape)}, got {tuple(grad_x_in.shape)}")
        grad_x_in = grad_x_in.to(x.dtype).contiguous()
    gx = torch.empty_like(x) if need_grad_x else x.new_empty((0,))
    ga = torch.empty((c, 16), device=x.device, dtype=torch.float32) if need_grad_alpha else x.new_empty((0,),
                                                                                                      dtype=torch.float32)
    with _guard(x):
        ws_bytes = _lib.load().lthc_read_bwd_workspace_bytes(b, g, c) if need_grad_alpha else 0
        ws = _workspace(ws_bytes, x.device) if need_grad_alpha else None
        _lib.call("lthc_read_bwd", x.data_ptr(), grad_z.data_ptr(), alpha.data_ptr(), _code(alpha, "read_bwd"),
                  _p(grad_x_in) if need_grad_x else None, gx.data_ptr() if need_grad_x else None, ga.data_ptr() if need_grad_alpha else None, _p(ws), ws_bytes,
                  b, g, c, _code(x, "read_bwd"), _stream(x))
    return gx, ga


@read_bwd.register_fake
def _(x, grad_z, alpha, need_grad_x, need_grad_alpha, grad_x_in=None):
    c = x.shape[-1]
    gx = torch.empty_like(x) if need_grad_x else x.new_empty((0,))
    ga = x.new_empty((c, 16), dtype=torch.float32) if need_grad_alpha else x.new_empty((0,), dtype=torch.float32)
    return gx, ga


def _read_setup(ctx, inputs, output):
    x, alpha = inputs
    ctx.save_for_backward(x, alpha)


def _read_backward(ctx, grad_z):
    x, alpha = ctx.saved_tensors
    need_x, need_a = ctx.needs_input_grad
    if not (need_x or need_a):
        return None, None
    gx, ga = read_bwd(x, grad_z, alpha, need_x, need_a)
    return (gx if need_x else None), (ga.to(alpha.dtype) if need_a else None)


read.register_autograd(_read_backward, setup_context=_read_setup)


# ---------------------------------------------------------------------------
# write / write_add / materialise: workspace -> residual
# ---------------------------------------------------------------------------
def _materialise_impl(x0: Tensor | None, dz: Sequence[Tensor], beta: Sequence[Tensor]) -> Tensor:
    L = len(dz)
    if L < 1 or L > MAX_LAYERS or len(beta) != L:
        raise ValueError(f"materialise: need 1..{MAX_LAYERS} layers with one beta each, got {L} dz / {len(beta)} beta")
    _require_cuda(*dz, *beta)
    b, g, c = _lo_geom(dz[0], "materialise")
    act = dz[0].dtype
    for t in dz:
        if tuple(t.shape) != (b, g * g, c):
            raise ValueError(f"materialise: every dz must be [{b},{g * g},{c}], got {tuple(t.shape)}")
    for w in beta:
        _check_weight(w, c, "materialise")
    wdt = beta[0].dtype
    dz = [t.to(act).contiguous() for t in dz]
    beta = [w.to(wdt).contiguous() for w in beta]
    if x0 is not None:
        _require_cuda(x0)
        if tuple(x0.shape) != (b, 4 * g, 4 * g, c):
            raise ValueError(f"materialise: expected x0 [{b},{4 * g},{4 * g},{c}], got {tuple(x0.shape)}")
        x0 = x0.to(act).contiguous()
    out = torch.empty((b, 4 * g, 4 * g, c), device=dz[0].device, dtype=act)
    with _guard(out):
        _lib.call("lthc_materialise_fwd", _p(x0), _lib.ptr_array([t.data_ptr() for t in dz]),
                  _lib.ptr_array([w.data_ptr() for w in beta]), _code(beta[0], "materialise"), L, out.data_ptr(), b, g,
                  c, _code(out, "materialise"), _stream(out))
    return out


@_custom_op("materialise")
def materialise(x0: Tensor, dz: list[Tensor], beta: list[Tensor]) -> Tensor:
    """X_L = X_0 + sum_l beta_l (.) dz_l in one pass, fp32 accumulation, one rounding.

    The B200 replacement of jit_thc::final_accumulate_b4_12_traceable
    (local_thc_triton_kernels.py:1669-1736).  Output dtype = x0 dtype."""
    if x0.dtype != dz[0].dtype:
        dz = [t.to(x0.dtype) for t in dz]
    return _materialise_impl(x0, dz, beta)


@materialise.register_fake
def _(x0, dz, beta):
    return torch.empty_like(x0)


@_custom_op("materialise_bwd")
def materialise_bwd(grad_out: Tensor, dz: list[Tensor], beta: list[Tensor], need_grad_dz: bool,
                    need_grad_beta: bool) -> tuple[list[Tensor], Tensor]:
    """grad_dz_l = sum_r beta_l grad_out (per cell); grad_beta = [L,C,16] fp32 sum grad_out*dz_l."""
    L = len(dz)
    _require_cuda(grad_out, *dz, *beta)
    b, g, c = _hi_geom(grad_out, "materialise_bwd")
    grad_out = grad_out.contiguous()
    act = grad_out.dtype
    dz = [t.to(act).contiguous() for t in dz]
    beta = [w.to(beta[0].dtype).contiguous() for w in beta]
    gdz = [torch.empty((b, g * g, c), device=grad_out.device, dtype=act) for _ in range(L)] if need_grad_dz else []
    gbeta = (torch.empty((L, c, 16), device=grad_out.device, dtype=torch.float32) if need_grad_beta
             else grad_out.new_empty((0,), dtype=torch.float32))
    with _guard(grad_out):
        ws_bytes = _lib.load().lthc_materialise_bwd_workspace_bytes(b, g, c, L) if need_grad_beta else 0
        ws = _workspace(ws_bytes, grad_out.device) if need_grad_beta else None
        _lib.call("lthc_materialise_bwd", grad_out.data_ptr(), _lib.ptr_array([t.data_ptr() for t in dz]),
                  _lib.ptr_array([w.data_ptr() for w in beta]), _code(beta[0], "materialise_bwd"), L,
                  _lib.ptr_array([t.data_ptr() for t in gdz]) if need_grad_dz else None,
                  gbeta.data_ptr() if need_grad_beta else None, _p(ws), ws_bytes, b, g, c,
                  _code(grad_out, "materialise_bwd"), _stream(grad_out))
    return gdz, gbeta


def materialise_bwd_uses_tensor_cores(B: int, G: int, C: int, L: int, dtype: torch.dtype) -> bool:
    """Whether materialise_bwd runs a [B, 4G, 4G, C] gradient of this dtype with L
    layers on the tensor cores (grad_dz then matches a sequential fp32 sum to one
    unit in the last place of the 16-bit output)."""
    return bool(_lib.load().lthc_materialise_bwd_uses_tensor_cores(B, G, C, L, _DTYPE_CODE[dtype]))


@materialise_bwd.register_fake
def _(grad_out, dz, beta, need_grad_dz, need_grad_beta):
    b, h, _, c = grad_out.shape
    g = h // 4
    gdz = [grad_out.new_empty((b, g * g, c)) for _ in dz] if need_grad_dz else []
    gbeta = (grad_out.new_empty((len(dz), c, 16), dtype=torch.float32) if need_grad_beta
             else grad_out.new_empty((0,), dtype=torch.float32))
    return gdz, gbeta


@_custom_op("materialise_grad_dz")
def materialise_grad_dz(grad_out: Tensor, beta: list[Tensor]) -> list[Tensor]:
    """grad_dz_l = sum_r beta_l grad_out per cell, alone: the weight-gradient half is
    not run and no update tensor is needed (the C call gets NULL for them)."""
    L = len(beta)
    if L < 1 or L > MAX_LAYERS:
        raise ValueError(f"materialise_grad_dz: need 1..{MAX_LAYERS} betas, got {L}")
    _require_cuda(grad_out, *beta)
    b, g, c = _hi_geom(grad_out, "materialise_grad_dz")
    for w in beta:
        _check_weight(w, c, "materialise_grad_dz")
    grad_out = grad_out.contiguous()
    beta = [w.to(beta[0].dtype).contiguous() for w in beta]
    gdz = [torch.empty((b, g * g, c), device=grad_out.device, dtype=grad_out.dtype) for _ in range(L)]
    with _guard(grad_out):
        _lib.call("lthc_materialise_bwd", grad_out.data_ptr(), None, _lib.ptr_array([w.data_ptr() for w in beta]),
                  _code(beta[0], "materialise_grad_dz"), L, _lib.ptr_array([t.data_ptr() for t in gdz]), None,
                  None, 0, b, g, c, _code(grad_out, "materialise_grad_dz"), _stream(grad_out))
    return gdz


@materialise_grad_dz.register_fake
def _(grad_out, beta):
    b, h, _, c = grad_out.shape
    return [grad_out.new_empty((b, (h // 4) ** 2, c)) for _ in beta]


@_custom_op("materialise_grad_beta")
def materialise_grad_beta(grad_out: Tensor, dz: list[Tensor]) -> Tensor:
    """grad_beta [L,C,16] fp32 = sum over cells of grad_out * dz_l, alone: no write
    weights are needed (the C call gets NULL for them)."""
    L = len(dz)
    if L < 1 or L > MAX_LAYERS:
        raise ValueError(f"materialise_grad_beta: need 1..{MAX_LAYERS} updates, got {L}")
    _require_cuda(grad_out, *dz)
    b, g, c = _hi_geom(grad_out, "materialise_grad_beta")
    for t in dz:
        if tuple(t.shape) != (b, g * g, c):
            raise ValueError(f"materialise_grad_beta: every dz must be [{b},{g * g},{c}], got {tuple(t.shape)}")
    grad_out = grad_out.contiguous()
    dz = [t.to(grad_out.dtype).contiguous() for t in dz]
    gbeta = torch.empty((L, c, 16), device=grad_out.device, dtype=torch.float32)
    with _guard(grad_out):
        ws_bytes = _lib.load().lthc_materialise_bwd_workspace_bytes(b, g, c, L)
        ws = _workspace(ws_bytes, grad_out.device)
        _lib.call("lthc_materialise_bwd", grad_out.data_ptr(), _lib.ptr_array([t.data_ptr() for t in dz]), None,
                  _lib.DTYPE_F32, L, None, gbeta.data_ptr(), ws.data_ptr(), ws_bytes, b, g, c,
                  _code(grad_out, "materialise_grad_beta"), _stream(grad_out))
    return gbeta


@materialise_grad_beta.register_fake
def _(grad_out, dz):
    return grad_out.new_empty((len(dz), grad_out.shape[-1], 16), dtype=torch.float32)


def _materialise_setup(ctx, inputs, output):
    x0, dz, beta = inputs
    ctx.save_for_backward(*dz, *beta)
    ctx.n_layers = len(dz)
    ctx.x0_dtype = x0.dtype


def _materialise_backward(ctx, grad_out):
    L = ctx.n_layers
    saved = ctx.saved_tensors
    dz, beta = list(saved[:L]), list(saved[L:])
    need_x0, need_dz, need_beta = ctx.needs_input_grad
    grad_out = grad_out.contiguous()
    gdz, gbeta = materialise_bwd(grad_out, dz, beta, bool(need_dz), bool(need_beta))
    # grad_x0 aliases grad_out, as _backward_final_accumulate_12 does
    # (local_thc_triton_kernels.py:1912)
    grad_dz = [t.to(d.dtype) for t, d in zip(gdz, dz)] if need_dz else None
    grad_beta = [gbeta[l].to(beta[l].dtype) for l in range(L)] if need_beta else None
    return (grad_out if need_x0 else None), grad_dz, grad_beta


materialise.register_autograd(_materialise_backward, setup_context=_materialise_setup)


@_custom_op("write")
def write(dz: Tensor, beta: Tensor) -> Tensor:
    """out[b,cell,r,c] = beta[c,r] dz[b,cell,c]  (LayerLocalWrite.write, local_thc.py:1261-1273)."""
    _require_cuda(dz, beta)
    b, g, c = _lo_geom(dz, "write")
    _check_weight(beta, c, "write")
    dz, beta = dz.contiguous(), beta.contiguous()
    out = torch.empty((b, 4 * g, 4 * g, c), device=dz.device, dtype=dz.dtype)
    with _guard(dz):
        _lib.call("lthc_write_fwd", dz.data_ptr(), beta.data_ptr(), _code(beta, "write"), out.data_ptr(), b, g, c,
                  _code(dz, "write"), _stream(dz))
    return out


@write.register_fake
def _(dz, beta):
    b, n, c = dz.shape
    g = math.isqrt(n)
    return dz.new_empty((b, 4 * g, 4 * g, c))


@_custom_op("write_bwd")
def write_bwd(grad_out: Tensor, dz: Tensor, beta: Tensor, need_grad_dz: bool, need_grad_beta: bool) -> tuple[Tensor, Tensor]:
    """grad_dz = sum_r beta grad_out (per cell); grad_beta = sum grad_out*dz (fp32 [C,16])."""
    _require_cuda(grad_out, dz, beta)
    b, g, c = _hi_geom(grad_out, "write_bwd")
    grad_out, dz, beta = grad_out.contiguous(), dz.to(grad_out.dtype).contiguous(), beta.contiguous()
    gdz = torch.empty((b, g * g, c), device=dz.device, dtype=grad_out.dtype) if need_grad_dz else dz.new_empty((0,))
    gb = (torch.empty((c, 16), device=dz.device, dtype=torch.float32) if need_grad_beta
          else dz.new_empty((0,), dtype=torch.float32))
    with _guard(dz):
        ws_bytes = _lib.load().lthc_write_bwd_workspace_bytes(b, g, c) if need_grad_beta else 0
        ws = _workspace(ws_bytes, dz.device) if need_grad_beta else None
        _lib.call("lthc_write_bwd", grad_out.data_ptr(), dz.data_ptr(), beta.data_ptr(), _code(beta, "write_bwd"),
                  gdz.data_ptr() if need_grad_dz else None, gb.data_ptr() if need_grad_beta else None, _p(ws),
                  ws_bytes, b, g, c, _code(grad_out, "write_bwd"), _stream(grad_out))
    return gdz, gb


@write_bwd.register_fake
def _(grad_out, dz, beta, need_grad_dz, need_grad_beta):
    c = grad_out.shape[-1]
    gdz = torch.empty_like(dz, dtype=grad_out.dtype) if need_grad_dz else dz.new_empty((0,))
    gb = dz.new_empty((c, 16), dtype=torch.float32) if need_grad_beta else dz.new_empty((0,), dtype=torch.float32)
    return gdz, gb


def _write_setup(ctx, inputs, output):
    dz, beta = inputs
    ctx.save_for_backward(dz, beta)


def _write_backward(ctx, grad_out):
    dz, beta = ctx.saved_tensors
    need_dz, need_beta = ctx.needs_input_grad
    if not (need_dz or need_beta):
        return None, None
    gdz, gb = write_bwd(grad_out, dz, beta, need_dz, need_beta)
    return (gdz.to(dz.dtype) if need_dz else None), (gb.to(beta.dtype) if need_beta else None)


write.register_autograd(_write_backward, setup_context=_write_setup)


@_custom_op("write_add")
def write_add(x_hi: Tensor, dz: Tensor, beta: Tensor) -> Tensor:
    """x_hi + write(dz)  (LayerLocalWrite.write_add, local_thc.py:1275-1276); fp32 sum, one rounding."""
    _require_cuda(x_hi, dz, beta)
    b, g, c = _hi_geom(x_hi, "write_add")
    if tuple(dz.shape) != (b, g * g, c):
        raise ValueError(f"write_add: expected dz [{b},{g * g},{c}], got {tuple(dz.shape)}")
    _check_weight(beta, c, "write_add")
    x_hi, dz, beta = x_hi.contiguous(), dz.to(x_hi.dtype).contiguous(), beta.contiguous()
    out = torch.empty_like(x_hi)
    with _guard(x_hi):
        _lib.call("lthc_write_add_fwd", x_hi.data_ptr(), dz.data_ptr(), beta.data_ptr(), _code(beta, "write_add"),
                  out.data_ptr(), b, g, c, _code(x_hi, "write_add"), _stream(x_hi))
    return out


@write_add.register_fake
def _(x_hi, dz, beta):
    return torch.empty_like(x_hi)


def _write_add_setup(ctx, inputs, output):
    x_hi, dz, beta = inputs
    ctx.save_for_backward(dz, beta)


def _write_add_backward(ctx, grad_out):
    dz, beta = ctx.saved_tensors
    need_x, need_dz, need_beta = ctx.needs_input_grad
    gdz = gb = None
    if need_dz or need_beta:
        gdz, gb = write_bwd(grad_out, dz, beta, need_dz, need_beta)
    return ((grad_out if need_x else None), (gdz.to(dz.dtype) if need_dz else None),
            (gb.to(beta.dtype) if need_beta else None))


write_add.register_autograd(_write_add_backward, setup_context=_write_add_setup)


# ---------------------------------------------------------------------------
# lazy shared-read recurrence  z' = z + gamma (.) dz,  gamma = sum_r alpha*beta
# ---------------------------------------------------------------------------
@_custom_op("lazy_update")
def lazy_update(z: Tensor, dz: Tensor, alpha: Tensor, beta: Tensor) -> Tensor:
    """Block.lazy_workspace_update with gamma_from_alpha (local_thc.py:1278-1283, 1325-1328)."""
    _require_cuda(z, dz, alpha, beta)
    if z.shape != dz.shape or z.dim() < 1:
        raise ValueError(f"lazy_update: z {tuple(z.shape)} and dz {tuple(dz.shape)} must match")
    c = z.shape[-1]
    _check_channels(c, "lazy_update")
    _check_weight(alpha, c, "lazy_update")
    _check_weight(beta, c, "lazy_update")
    z, dz, alpha, beta = z.contiguous(), dz.to(z.dtype).contiguous(), alpha.contiguous(), beta.contiguous()
    out = torch.empty_like(z)
    n = z.numel() // c
    with _guard(z):
        _lib.call("lthc_lazy_update_fwd", z.data_ptr(), dz.data_ptr(), alpha.data_ptr(), _code(alpha, "lazy_update"),
                  beta.data_ptr(), _code(beta, "lazy_update"), out.data_ptr(), n, c, _code(z, "lazy_update"),
                  _stream(z))
    return out


@lazy_update.register_fake
def _(z, dz, alpha, beta):
    return torch.empty_like(z)


@_custom_op("lazy_update_bwd")
def lazy_update_bwd(grad_z_out: Tensor, dz: Tensor, alpha: Tensor, beta: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """(grad_dz, grad_alpha fp32 [C,16], grad_beta fp32 [C,16]); grad_z is grad_z_out itself."""
    _require_cuda(grad_z_out, dz, alpha, beta)
    c = grad_z_out.shape[-1]
    g, dz = grad_z_out.contiguous(), dz.to(grad_z_out.dtype).contiguous()
    alpha, beta = alpha.contiguous(), beta.contiguous()
    n = g.numel() // c
    gdz = torch.empty_like(g)
    ga = torch.empty((c, 16), device=g.device, dtype=torch.float32)
    gb = torch.empty((c, 16), device=g.device, dtype=torch.float32)
    with _guard(g):
        ws_bytes = _lib.load().lthc_lazy_update_bwd_workspace_bytes(n, c)
        ws = _workspace(ws_bytes, g.device)
        _lib.call("lthc_lazy_update_bwd", g.data_ptr(), dz.data_ptr(), alpha.data_ptr(),
                  _code(alpha, "lazy_update_bwd"), beta.data_ptr(), _code(beta, "lazy_update_bwd"), gdz.data_ptr(),
                  ga.data_ptr(), gb.data_ptr(), ws.data_ptr(), ws_bytes, n, c, _code(g, "lazy_update_bwd"), _stream(g))
    return gdz, ga, gb


@lazy_update_bwd.register_fake
def _(grad_z_out, dz, alpha, beta):
    c = grad_z_out.shape[-1]
    return (torch.empty_like(grad_z_out), grad_z_out.new_empty((c, 16), dtype=torch.float32),
            grad_z_out.new_empty((c, 16), dtype=torch.float32))


def _lazy_setup(ctx, inputs, output):
    z, dz, alpha, beta = inputs
    ctx.save_for_backward(dz, alpha, beta)


def _lazy_backward(ctx, grad_out):
    dz, alpha, beta = ctx.saved_tensors
    need_z, need_dz, need_a, need_b = ctx.needs_input_grad
    gdz, ga, gb = lazy_update_bwd(grad_out, dz, alpha, beta)
    return ((grad_out if need_z else None), (gdz.to(dz.dtype) if need_dz else None),
            (ga.to(alpha.dtype) if need_a else None), (gb.to(beta.dtype) if need_b else None))


lazy_update.register_autograd(_lazy_backward, setup_context=_lazy_setup)


# ---------------------------------------------------------------------------
# weight gradient  grad_w[l,c,r] = sum_cells high[cell,r,c] * low_l[cell,c]
# ---------------------------------------------------------------------------
@_custom_op("weight_grad")
def weight_grad(high: Tensor, low: list[Tensor]) -> Tensor:
    """[L,C,16] fp32, reduced in a fixed order (replaces the atomics of
    _cell_weight_grad_kernel, local_thc_triton_kernels.py:167-199)."""
    _require_cuda(high, *low)
    b, g, c = _hi_geom(high, "weight_grad")
    L = len(low)
    if L < 1 or L > MAX_LAYERS:
        raise ValueError(f"weight_grad: need 1..{MAX_LAYERS} workspace tensors, got {L}")
    high = high.contiguous()
    low = [t.to(high.dtype).contiguous() for t in low]
    for t in low:
        if tuple(t.shape) != (b, g * g, c):
            raise ValueError(f"weight_grad: expected low [{b},{g * g},{c}], got {tuple(t.shape)}")
    out = torch.empty((L, c, 16), device=high.device, dtype=torch.float32)
    with _guard(high):
        ws_bytes = _lib.load().lthc_weight_grad_workspace_bytes(b, g, c, L)
        ws = _workspace(ws_bytes, high.device)
        _lib.call("lthc_weight_grad", high.data_ptr(), _lib.ptr_array([t.data_ptr() for t in low]), L, out.data_ptr(),
                  ws.data_ptr(), ws_bytes, b, g, c, _code(high, "weight_grad"), _stream(high))
    return out


@weight_grad.register_fake
def _(high, low):
    return high.new_empty((len(low), high.shape[-1], 16), dtype=torch.float32)


# ---------------------------------------------------------------------------
# branch epilogue fused with the lazy update
# (WorkspaceSharedAdaLNBranch.forward's output sum, local_thc.py:318-323, then
# lazy_workspace_update, :1325-1328)
# ---------------------------------------------------------------------------
def _branch_geom(z: Tensor, dz_attn: Tensor, mlp_out: Tensor, gate: Tensor, what: str) -> tuple[int, int, int]:
    if z.dim() != 3:
        raise ValueError(f"{what}: expected workspace rows [B,T,C], got {tuple(z.shape)}")
    b, t, c = z.shape
    _check_channels(c, what)
    for name, u in (("dz_attn", dz_attn), ("mlp_out", mlp_out)):
        if u.shape != z.shape:
            raise ValueError(f"{what}: {name} {tuple(u.shape)} must match z {tuple(z.shape)}")
    if tuple(gate.shape) != (b, c):
        raise ValueError(f"{what}: expected gate [{b},{c}], got {tuple(gate.shape)}")
    for u in (dz_attn, mlp_out, gate):
        if u.dtype != z.dtype:
            raise ValueError(f"{what}: all activations must share z's dtype {z.dtype}, got {u.dtype}")
    return b, t, c


def _gate_rows(gate: Tensor) -> tuple[Tensor, int]:
    """gate and its row stride; a chunk of t6 (rows 16-byte aligned) passes without a copy."""
    c = gate.shape[1]
    es = gate.element_size()
    if (gate.stride(1) == 1 and gate.stride(0) >= c and gate.stride(0) % 8 == 0 and (gate.stride(0) * es) % 16 == 0
            and gate.data_ptr() % 16 == 0):
        return gate, gate.stride(0)
    return gate.contiguous(), c


@_custom_op("branch_lazy_update")
def branch_lazy_update(z: Tensor, dz_attn: Tensor, mlp_out: Tensor, gate: Tensor, alpha: Tensor,
                       beta: Tensor) -> tuple[Tensor, Tensor]:
    """(dz, z_next): dz = dz_attn + gate (.) mlp_out, z_next = z + gamma (.) dz."""
    _require_cuda(z, dz_attn, mlp_out, gate, alpha, beta)
    b, t, c = _branch_geom(z, dz_attn, mlp_out, gate, "branch_lazy_update")
    _check_weight(alpha, c, "branch_lazy_update")
    _check_weight(beta, c, "branch_lazy_update")
    z, dz_attn, mlp_out = z.contiguous(), dz_attn.contiguous(), mlp_out.contiguous()
    alpha, beta = alpha.contiguous(), beta.contiguous()
    gate, gs = _gate_rows(gate)
    dz, zn = torch.empty_like(z), torch.empty_like(z)
    with _guard(z):
        _lib.call("lthc_branch_lazy_fwd", z.data_ptr(), dz_attn.data_ptr(), mlp_out.data_ptr(), gate.data_ptr(), gs,
                  alpha.data_ptr(), _code(alpha, "branch_lazy_update"), beta.data_ptr(), _code(beta, "branch_lazy_update"),
                  dz.data_ptr(), zn.data_ptr(), b, t, c, _code(z, "branch_lazy_update"), _stream(z))
    return dz, zn


@branch_lazy_update.register_fake
def _(z, dz_attn, mlp_out, gate, alpha, beta):
    return torch.empty_like(z), torch.empty_like(z)


@_custom_op("branch_lazy_update_bwd")
def branch_lazy_update_bwd(grad_dz: Tensor | None, grad_z_next: Tensor, dz: Tensor, mlp_out: Tensor, gate: Tensor,
                           alpha: Tensor, beta: Tensor) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """(grad dz_attn, grad mlp_out, grad gate fp32 [B,C], grad alpha fp32, grad beta fp32)."""
    _require_cuda(grad_z_next, dz, mlp_out, gate, alpha, beta)
    b, t, c = _branch_geom(dz, dz, mlp_out, gate, "branch_lazy_update_bwd")
    gz = grad_z_next.to(dz.dtype).contiguous()
    gd = grad_dz.to(dz.dtype).contiguous() if grad_dz is not None else None
    dz, mlp_out, alpha, beta = dz.contiguous(), mlp_out.contiguous(), alpha.contiguous(), beta.contiguous()
    gate, gs = _gate_rows(gate)
    g_attn, g_mlp = torch.empty_like(dz), torch.empty_like(dz)
    g_gate = torch.empty((b, c), device=dz.device, dtype=torch.float32)
    ga = torch.empty((c, 16), device=dz.device, dtype=torch.float32)
    gb = torch.empty((c, 16), device=dz.device, dtype=torch.float32)
    with _guard(dz):
        ws_bytes = _lib.load().lthc_branch_lazy_bwd_workspace_bytes(b, t, c)
        ws = _workspace(ws_bytes, dz.device)
        _lib.call("lthc_branch_lazy_bwd", _p(gd), gz.data_ptr(), dz.data_ptr(), mlp_out.data_ptr(), gate.data_ptr(), gs,
                  alpha.data_ptr(), _code(alpha, "branch_lazy_update_bwd"), beta.data_ptr(),
                  _code(beta, "branch_lazy_update_bwd"), g_attn.data_ptr(), g_mlp.data_ptr(), g_gate.data_ptr(),
                  ga.data_ptr(), gb.data_ptr(), ws.data_ptr(), ws_bytes, b, t, c, _code(dz, "branch_lazy_update_bwd"),
                  _stream(dz))
    return g_attn, g_mlp, g_gate, ga, gb


@branch_lazy_update_bwd.register_fake
def _(grad_dz, grad_z_next, dz, mlp_out, gate, alpha, beta):
    b, t, c = dz.shape
    f32 = dict(dtype=torch.float32)
    return (torch.empty_like(dz), torch.empty_like(dz), dz.new_empty((b, c), **f32), dz.new_empty((c, 16), **f32),
            dz.new_empty((c, 16), **f32))


def _branch_setup(ctx, inputs, output):
    z, dz_attn, mlp_out, gate, alpha, beta = inputs
    dz, _ = output
    ctx.save_for_backward(dz, mlp_out, gate, alpha, beta)


def _branch_backward(ctx, grad_dz, grad_z_next):
    dz, mlp_out, gate, alpha, beta = ctx.saved_tensors
    need_z, need_attn, need_mlp, need_gate, need_a, need_b = ctx.needs_input_grad
    if grad_z_next is None:
        grad_z_next = torch.zeros_like(dz)
    g_attn, g_mlp, g_gate, ga, gb = branch_lazy_update_bwd(grad_dz, grad_z_next, dz, mlp_out, gate, alpha, beta)
    return ((grad_z_next if need_z else None), (g_attn if need_attn else None), (g_mlp if need_mlp else None),
            (g_gate.to(gate.dtype) if need_gate else None), (ga.to(alpha.dtype) if need_a else None),
            (gb.to(beta.dtype) if need_b else None))


branch_lazy_update.register_autograd(_branch_backward, setup_context=_branch_setup)


# ---------------------------------------------------------------------------
# patch embedding fused with the shared read (tensor cores)
# (BottleneckPatchEmbedNHWC.forward, local_thc.py:64-89, then SharedLocalRead.read,
# :1211-1223)
# ---------------------------------------------------------------------------
EMBED_CHUNK = 256
EMBED_TILE_COLS = 32


def embed_supported(img: Tensor, w1: Tensor, w2: Tensor) -> bool:
    """Shapes the fused kernel takes: 4x4/4 patches of 1..4 channels into a 128-wide
    bottleneck, C a multiple of 256, a token grid side that is a multiple of 32."""
    if img.dim() != 4 or w1.dim() != 4 or w2.dim() != 4:
        return False
    b, cin, s, s2 = img.shape
    return (s == s2 and s % (4 * EMBED_TILE_COLS) == 0 and tuple(w1.shape) == (128, cin, 4, 4) and 1 <= cin <= 4
            and w2.shape[1] == 128 and tuple(w2.shape[2:]) == (1, 1) and w2.shape[0] % EMBED_CHUNK == 0)


@_custom_op("patch_embed_read")
def patch_embed_read(img: Tensor, w1: Tensor, w2: Tensor, b2: Tensor, alpha: Tensor) -> tuple[Tensor, Tensor]:
    """(X0 [B,H,H,C] bf16, Z [B,(H/4)^2,C] bf16): both convolutions in bf16 with fp32
    accumulation on the tensor cores, then the read of X0 with alpha."""
    _require_cuda(img, w1, w2, b2, alpha)
    if not embed_supported(img, w1, w2):
        raise ValueError(f"patch_embed_read: unsupported shapes img {tuple(img.shape)}, w1 {tuple(w1.shape)}, "
                         f"w2 {tuple(w2.shape)}")
    b, cin, s, _ = img.shape
    c = w2.shape[0]
    h = s // 4
    if tuple(b2.shape) != (c,) or tuple(alpha.shape) != (c, 16):
        raise ValueError(f"patch_embed_read: expected bias [{c}] and alpha [{c},16]")
    if img.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError(f"patch_embed_read: image dtype {img.dtype} (float32 or bfloat16)")
    bf = torch.bfloat16
    img = img.contiguous()
    w1b = w1.to(bf).reshape(128, cin * 16).contiguous()
    w2b = w2.to(bf).reshape(c, 128).contiguous()
    b2b, ab = b2.to(bf).contiguous(), alpha.to(bf).contiguous()
    x0 = torch.empty((b, h, h, c), device=img.device, dtype=bf)
    z = torch.empty((b, (h // 4) ** 2, c), device=img.device, dtype=bf)
    with _guard(img):
        _lib.call("lthc_patch_embed_read_fwd", img.data_ptr(), _code(img, "patch_embed_read"), w1b.data_ptr(),
                  w2b.data_ptr(), b2b.data_ptr(), ab.data_ptr(), x0.data_ptr(), z.data_ptr(), b, cin, h, c,
                  _stream(img))
    return x0, z


@patch_embed_read.register_fake
def _(img, w1, w2, b2, alpha):
    b, _, s, _ = img.shape
    c, h = w2.shape[0], s // 4
    bf = torch.bfloat16
    return img.new_empty((b, h, h, c), dtype=bf), img.new_empty((b, (h // 4) ** 2, c), dtype=bf)


def _embed_setup(ctx, inputs, output):
    img, w1, w2, b2, alpha = inputs
    x0, _ = output
    ctx.save_for_backward(img, w1, w2, alpha, x0)
    ctx.b2_dtype = b2.dtype


def _embed_backward(ctx, g_x0, g_z):
    """The read's backward with the gradient X0 already receives from the
    materialisation as its base: grad X0 = g_x0 + alpha (.) bcast(g_z) in one
    write-family pass (no separate read-backward output and add), grad alpha from
    the same call's weight-gradient pass; then the two convolutions' backward as
    library GEMMs on the bf16 operands (h1 recomputed)."""
    img, w1, w2, alpha, x0 = ctx.saved_tensors
    need_img, need_w1, need_w2, need_b2, need_a = ctx.needs_input_grad
    bf = torch.bfloat16
    b, cin, s, _ = img.shape
    c, h = w2.shape[0], s // 4
    gx = g_x0 if g_x0 is not None else torch.zeros_like(x0)
    ga = None
    if g_z is not None:
        gx, ga = read_bwd(x0, g_z.to(bf), alpha.to(bf), True, need_a, g_x0.to(bf) if g_x0 is not None else None)
    g2 = gx.to(bf).reshape(-1, c)                                              # [tokens, C]
    patches = (img.to(bf).reshape(b, cin, h, 4, h, 4).permute(0, 2, 4, 1, 3, 5).reshape(-1, cin * 16))
    w1b = w1.to(bf).reshape(128, cin * 16)
    w2b = w2.to(bf).reshape(c, 128)
    h1 = patches @ w1b.t()                                                     # [tokens, 128] bf16
    gw2 = (g2.t() @ h1).reshape(w2.shape).to(w2.dtype) if need_w2 else None
    gb2 = g2.float().sum(0).to(ctx.b2_dtype) if need_b2 else None
    gw1 = None
    if need_w1 or need_img:
        gh1 = g2 @ w2b                                                         # [tokens, 128]
        gw1 = (gh1.t() @ patches).reshape(w1.shape).to(w1.dtype) if need_w1 else None
    gimg = None
    if need_img:
        gp = (gh1 @ w1b).float()                                               # [tokens, cin*16]
        gimg = gp.reshape(b, h, h, cin, 4, 4).permute(0, 3, 1, 4, 2, 5).reshape(img.shape).to(img.dtype)
    return gimg, gw1, gw2, gb2, (ga.to(alpha.dtype) if (need_a and ga is not None) else None)


patch_embed_read.register_autograd(_embed_backward, setup_context=_embed_setup)


# ---------------------------------------------------------------------------
# final-layer prologue  m = modulate(RMSNorm(x), shift, scale)
# (FinalLayerSharedAdaLN.forward, local_thc.py:865-873; RMSNorm,
# jit_shared_adaln.py:20-30; modulate, local_thc.py:37-38)
# ---------------------------------------------------------------------------
FINAL_MAX_CHANNELS = 1024


def _final_geom(x: Tensor, weight: Tensor, shift: Tensor, scale: Tensor, what: str) -> tuple[int, int, int]:
    if x.dim() != 3:
        raise ValueError(f"{what}: expected tokens [B,T,C], got {tuple(x.shape)}")
    b, t, c = x.shape
    if c % 8 != 0 or c < 8 or c > FINAL_MAX_CHANNELS:
        raise ValueError(f"{what}: channel count {c} must be a multiple of 8 in [8, {FINAL_MAX_CHANNELS}]")
    if tuple(weight.shape) != (c,):
        raise ValueError(f"{what}: expected norm weight [{c}], got {tuple(weight.shape)}")
    for name, m in (("shift", shift), ("scale", scale)):
        if tuple(m.shape) != (b, c):
            raise ValueError(f"{what}: expected {name} [{b},{c}], got {tuple(m.shape)}")
        if m.dtype != x.dtype:
            raise ValueError(f"{what}: {name} dtype {m.dtype} differs from the activation dtype {x.dtype}")
    return b, t, c


def _mod_rows(shift: Tensor, scale: Tensor) -> tuple[Tensor, Tensor, int]:
    """shift / scale and their common row stride; the two halves of
    ``t2.chunk(2, dim=1)`` pass through without a copy."""
    c = shift.shape[1]
    if (shift.stride(1) == 1 and scale.stride(1) == 1 and shift.stride(0) == scale.stride(0)
            and shift.stride(0) >= c):
        return shift, scale, shift.stride(0)
    return shift.contiguous(), scale.contiguous(), c


@_custom_op("final_norm_modulate")
def final_norm_modulate(x: Tensor, weight: Tensor, shift: Tensor, scale: Tensor, eps: float) -> Tensor:
    """modulate(RMSNorm(x) with weight and eps, shift, scale) over tokens [B,T,C]."""
    _require_cuda(x, weight, shift, scale)
    b, t, c = _final_geom(x, weight, shift, scale, "final_norm_modulate")
    x, weight = x.contiguous(), weight.contiguous()
    sh, sc, stride = _mod_rows(shift, scale)
    out = torch.empty_like(x)
    with _guard(x):
        _lib.call("lthc_final_norm_modulate_fwd", x.data_ptr(), weight.data_ptr(), _code(weight, "norm weight"),
                  sh.data_ptr(), sc.data_ptr(), stride, out.data_ptr(), b, t, c, float(eps),
                  _code(x, "final_norm_modulate"), _stream(x))
    return out


@final_norm_modulate.register_fake
def _(x, weight, shift, scale, eps):
    return torch.empty_like(x)


@_custom_op("final_norm_modulate_bwd")
def final_norm_modulate_bwd(grad_out: Tensor, x: Tensor, weight: Tensor, scale: Tensor,
                            eps: float) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """(grad_x, grad_weight fp32 [C], grad_shift fp32 [B,C], grad_scale fp32 [B,C])."""
    _require_cuda(grad_out, x, weight, scale)
    b, t, c = _final_geom(x, weight, scale, scale, "final_norm_modulate_bwd")
    x, weight, g = x.contiguous(), weight.contiguous(), grad_out.to(x.dtype).contiguous()
    _, sc, stride = _mod_rows(scale, scale)
    gx = torch.empty_like(x)
    gw = torch.empty((c,), device=x.device, dtype=torch.float32)
    gsh = torch.empty((b, c), device=x.device, dtype=torch.float32)
    gsc = torch.empty((b, c), device=x.device, dtype=torch.float32)
    with _guard(x):
        ws_bytes = _lib.load().lthc_final_norm_modulate_bwd_workspace_bytes(b, t, c)
        ws = _workspace(ws_bytes, x.device)
        _lib.call("lthc_final_norm_modulate_bwd", x.data_ptr(), weight.data_ptr(), _code(weight, "norm weight"),
                  sc.data_ptr(), stride, g.data_ptr(), gx.data_ptr(), gw.data_ptr(), gsh.data_ptr(), gsc.data_ptr(),
                  ws.data_ptr(), ws_bytes, b, t, c, float(eps), _code(x, "final_norm_modulate_bwd"), _stream(x))
    return gx, gw, gsh, gsc


@final_norm_modulate_bwd.register_fake
def _(grad_out, x, weight, scale, eps):
    b, _, c = x.shape
    f32 = dict(dtype=torch.float32)
    return torch.empty_like(x), x.new_empty((c,), **f32), x.new_empty((b, c), **f32), x.new_empty((b, c), **f32)


def _final_setup(ctx, inputs, output):
    x, weight, shift, scale, eps = inputs
    ctx.eps = eps
    ctx.shift_dtype = shift.dtype
    ctx.save_for_backward(x, weight, scale)


def _final_backward(ctx, grad_out):
    x, weight, scale = ctx.saved_tensors
    need_x, need_w, need_sh, need_sc, _ = ctx.needs_input_grad
    gx, gw, gsh, gsc = final_norm_modulate_bwd(grad_out, x, weight, scale, ctx.eps)
    return ((gx if need_x else None), (gw.to(weight.dtype) if need_w else None),
            (gsh.to(ctx.shift_dtype) if need_sh else None), (gsc.to(scale.dtype) if need_sc else None), None)


final_norm_modulate.register_autograd(_final_backward, setup_context=_final_setup)




# ---------------------------------------------------------------------------
# Mirrors of the reference jit_thc:: Triton op surface (same names and argument
# order; "local_write" = read and "local_read" = write are that file's legacy
# names, local_thc_triton_kernels.py:2673-2723).
# ---------------------------------------------------------------------------
def final_accumulate_b4_12_traceable(x0: Tensor, *dz_and_beta: Tensor) -> Tensor:
    """jit_thc::final_accumulate_b4_12_traceable(x0, dz0..dz11, beta0..beta11) (:1669-1736)."""
    if len(dz_and_beta) != 24:
        raise ValueError(f"expected 12 dz and 12 beta tensors, got {len(dz_and_beta)} tensors")
    return materialise(x0, list(dz_and_beta[:12]), list(dz_and_beta[12:]))


def final_accumulate_b4_traceable(x0: Tensor, dz_stack: Tensor, beta_stack: Tensor) -> Tensor:
    """jit_thc::final_accumulate_b4_traceable(x0, dz[L,B,256,C], beta[L,C,16]) (:1578-1598)."""
    return materialise(x0, list(dz_stack.unbind(0)), list(beta_stack.unbind(0)))


def final_accumulate_b4_12_grad_dz_ptr_traceable(grad_out: Tensor, *betas: Tensor) -> Tensor:
    """jit_thc::final_accumulate_b4_12_grad_dz_ptr -> [12,B,256,C] (:1800-1845)."""
    if len(betas) != 12:
        raise ValueError(f"expected 12 beta tensors, got {len(betas)}")
    return torch.stack(materialise_grad_dz(grad_out, list(betas)))


def final_accumulate_b4_12_grad_beta_ptr_traceable(grad_out: Tensor, *dzs: Tensor) -> Tensor:
    """jit_thc::final_accumulate_b4_12_grad_beta_ptr -> [12,C,16] fp32 (:1848-1894)."""
    if len(dzs) != 12:
        raise ValueError(f"expected 12 dz tensors, got {len(dzs)}")
    return materialise_grad_beta(grad_out, list(dzs))


def local_write_traceable(x: Tensor, weight: Tensor) -> Tensor:
    """jit_thc::local_write_traceable = the read (:2673-2683)."""
    return read(x, weight)


def local_read_traceable(z: Tensor, weight: Tensor) -> Tensor:
    """jit_thc::local_read_traceable = the write (:2686-2696)."""
    return write(z, weight)


def local_read_add_traceable(z: Tensor, weight: Tensor, x: Tensor) -> Tensor:
    """jit_thc::local_read_add_traceable(z, weight, x) = x + write(z) (:2713-2723)."""
    return write_add(x, z, weight)


def local_weight_grad_traceable(high: Tensor, low: Tensor) -> Tensor:
    """jit_thc::local_weight_grad_traceable(high, low) -> [C,16] fp32 (:2699-2710)."""
    return weight_grad(high, [low])[0]


__all__ = [
    "read", "read_bwd", "write", "write_bwd", "write_add", "materialise", "materialise_bwd", "materialise_grad_dz",
    "materialise_grad_beta", "lazy_update",
    "lazy_update_bwd", "weight_grad", "final_accumulate_b4_12_traceable", "final_accumulate_b4_traceable",
    "final_accumulate_b4_12_grad_dz_ptr_traceable", "final_accumulate_b4_12_grad_beta_ptr_traceable",
    "local_write_traceable", "local_read_traceable", "local_read_add_traceable", "local_weight_grad_traceable",
]
