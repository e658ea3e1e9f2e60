"""ctypes front end of the C oracle, on CPU torch tensors.

TEST INFRASTRUCTURE ONLY: the checker for the CUDA kernels and the timed CPU
baseline.  Tensors are contiguous CPU tensors of dtype float32, bfloat16 or
float16 (torch is used here only as a container; all arithmetic is in
``lthc_oracle.c``).  Each function names the reference code it restates
(paths inside tongtongliang/flowmatching_lthc).
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_void_p
from typing import Sequence

import torch

from .build_oracle import OUT, build

_DT = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = build()
        L = ctypes.CDLL(str(path))
        i64, p, i = c_int64, c_void_p, c_int
        sig = {
            "oracle_read": [p, p, i, p, i64, i64, i64, i],
            "oracle_write": [p, p, i, p, i64, i64, i64, i],
            "oracle_write_add": [p, p, p, i, p, i64, i64, i64, i],
            "oracle_materialise": [p, ctypes.POINTER(p), ctypes.POINTER(p), i, i, p, i64, i64, i64, i],
            "oracle_materialise_bwd": [p, ctypes.POINTER(p), ctypes.POINTER(p), i, i, ctypes.POINTER(p), p, i64, i64,
                                       i64, i],
            "oracle_weight_grad": [p, ctypes.POINTER(p), i, p, i64, i64, i64, i],
            "oracle_lazy_fwd": [p, p, p, i, p, i, p, i64, i64, i],
            "oracle_lazy_bwd": [p, p, p, i, p, i, p, p, p, i64, i64, i],
            "oracle_final_fwd": [p, p, i, p, p, i64, p, i64, i64, i64, c_float, i],
            "oracle_final_bwd": [p, p, i, p, i64, p, p, p, p, p, i64, i64, i64, c_float, i],
            "oracle_branch_fwd": [p, p, p, p, i64, p, i, p, i, p, p, i64, i64, i64, i],
            "oracle_branch_bwd": [p, p, p, p, p, i64, p, i, p, i, p, p, p, p, p, i64, i64, i64, i],
            "oracle_num_threads": [],
            "oracle_set_num_threads": [i],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = c_int if name == "oracle_num_threads" else None
        _lib = L
    return _lib


def _c(t: torch.Tensor) -> torch.Tensor:
    if t.device.type != "cpu":
        raise ValueError("the oracle runs on CPU tensors")
    if t.dtype not in _DT:
        raise ValueError(f"unsupported dtype {t.dtype}")
    return t.contiguous()


def _p(t: torch.Tensor | None) -> c_void_p:
    return c_void_p(t.data_ptr()) if t is not None else c_void_p(0)


def _parr(ts: Sequence[torch.Tensor]):
    return (c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def _geom_hi(x: torch.Tensor) -> tuple[int, int, int]:
    b, h, w, c = x.shape
    if h != w or h % 4:
        raise ValueError(f"expected [B,4G,4G,C], got {tuple(x.shape)}")
    return b, h // 4, c


def _geom_lo(z: torch.Tensor) -> tuple[int, int, int]:
    b, n, c = z.shape
    g = int(round(n ** 0.5))
    if g * g != n:
        raise ValueError(f"workspace token count {n} is not square")
    return b, g, c


def num_threads() -> int:
    return int(lib().oracle_num_threads())


def set_num_threads(n: int) -> None:
    lib().oracle_set_num_threads(int(n))


def read(x: torch.Tensor, alpha: torch.Tensor) -> torch.Tensor:
    """SharedLocalRead.read (local_thc.py:1211-1223): z = sum_r alpha[c,r] x[cell,r,c]."""
    x, alpha = _c(x), _c(alpha)
    b, g, c = _geom_hi(x)
    z = torch.empty(b, g * g, c, dtype=x.dtype)
    lib().oracle_read(_p(x), _p(alpha), _DT[alpha.dtype], _p(z), b, g, c, _DT[x.dtype])
    return z


def write(dz: torch.Tensor, beta: torch.Tensor) -> torch.Tensor:
    """LayerLocalWrite.write (local_thc.py:1261-1273): out[cell,r,c] = beta[c,r] dz[cell,c]."""
    dz, beta = _c(dz), _c(beta)
    b, g, c = _geom_lo(dz)
    out = torch.empty(b, 4 * g, 4 * g, c, dtype=dz.dtype)
    lib().oracle_write(_p(dz), _p(beta), _DT[beta.dtype], _p(out), b, g, c, _DT[dz.dtype])
    return out


def write_add(x: torch.Tensor, dz: torch.Tensor, beta: torch.Tensor) -> torch.Tensor:
    """LayerLocalWrite.write_add (local_thc.py:1275-1276): x + write(dz)."""
    x, dz, beta = _c(x), _c(dz), _c(beta)
    b, g, c = _geom_hi(x)
    out = torch.empty_like(x)
    lib().oracle_write_add(_p(x), _p(dz), _p(beta), _DT[beta.dtype], _p(out), b, g, c, _DT[x.dtype])
    return out


def materialise(x0: torch.Tensor | None, dz: Sequence[torch.Tensor], beta: Sequence[torch.Tensor]) -> torch.Tensor:
    """X_L = X_0 + sum_l beta_l (.) dz_l, one rounding (local_thc_triton_kernels.py:317-405)."""
    dz = [_c(t) for t in dz]
    beta = [_c(t) for t in beta]
    b, g, c = _geom_lo(dz[0])
    if x0 is not None:
        x0 = _c(x0)
    out = torch.empty(b, 4 * g, 4 * g, c, dtype=dz[0].dtype)
    lib().oracle_materialise(_p(x0), _parr(dz), _parr(beta), _DT[beta[0].dtype], len(dz), _p(out), b, g, c,
                             _DT[dz[0].dtype])
    return out


def materialise_bwd(gout: torch.Tensor, dz: Sequence[torch.Tensor], beta: Sequence[torch.Tensor]):
    """_backward_final_accumulate_12 (local_thc_triton_kernels.py:1897-1912).

    Returns (grad_dz list, grad_beta float32 [L,C,16]); grad_x0 is gout itself."""
    gout = _c(gout)
    dz = [_c(t) for t in dz]
    beta = [_c(t) for t in beta]
    b, g, c = _geom_hi(gout)
    L = len(dz)
    gdz = [torch.empty(b, g * g, c, dtype=gout.dtype) for _ in range(L)]
    gw = torch.empty(L, c, 16, dtype=torch.float32)
    lib().oracle_materialise_bwd(_p(gout), _parr(dz), _parr(beta), _DT[beta[0].dtype], L, _parr(gdz), _p(gw), b, g,
                                 c, _DT[gout.dtype])
    return gdz, gw


def weight_grad(high: torch.Tensor, low: Sequence[torch.Tensor]) -> torch.Tensor:
    """_cell_weight_grad_kernel (local_thc_triton_kernels.py:167-199): [L,C,16] float32."""
    high = _c(high)
    low = [_c(t) for t in low]
    b, g, c = _geom_hi(high)
    gw = torch.empty(len(low), c, 16, dtype=torch.float32)
    lib().oracle_weight_grad(_p(high), _parr(low), len(low), _p(gw), b, g, c, _DT[high.dtype])
    return gw


def lazy_fwd(z: torch.Tensor, dz: torch.Tensor, alpha: torch.Tensor, beta: torch.Tensor) -> torch.Tensor:
    """lazy_workspace_update (local_thc.py:1325-1328) with gamma_from_alpha (:1278-1283)."""
    z, dz, alpha, beta = _c(z), _c(dz), _c(alpha), _c(beta)
    c = z.shape[-1]
    n = z.numel() // c
    out = torch.empty_like(z)
    lib().oracle_lazy_fwd(_p(z), _p(dz), _p(alpha), _DT[alpha.dtype], _p(beta), _DT[beta.dtype], _p(out), n, c,
                          _DT[z.dtype])
    return out


def lazy_bwd(gzo: torch.Tensor, dz: torch.Tensor, alpha: torch.Tensor, beta: torch.Tensor):
    """Autograd of lazy_workspace_update: (grad_dz, grad_alpha fp32, grad_beta fp32)."""
    gzo, dz, alpha, beta = _c(gzo), _c(dz), _c(alpha), _c(beta)
    c = gzo.shape[-1]
    n = gzo.numel() // c
    gdz = torch.empty_like(gzo)
    ga = torch.empty(c, 16, dtype=torch.float32)
    gb = torch.empty(c, 16, dtype=torch.float32)
    lib().oracle_lazy_bwd(_p(gzo), _p(dz), _p(alpha), _DT[alpha.dtype], _p(beta), _DT[beta.dtype], _p(gdz), _p(ga),
                          _p(gb), n, c, _DT[gzo.dtype])
    return gdz, ga, gb


def _mod(shift: torch.Tensor, scale: torch.Tensor):
    shift, scale = _c(shift), _c(scale)
    return shift, scale, shift.shape[1]


def final_fwd(x: torch.Tensor, weight: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor,
              eps: float) -> torch.Tensor:
    """FinalLayerSharedAdaLN.forward without its Linear (local_thc.py:865-873): modulate(RMSNorm(x))."""
    x, weight = _c(x), _c(weight)
    shift, scale, ms = _mod(shift, scale)
    b, t, c = x.shape
    out = torch.empty_like(x)
    lib().oracle_final_fwd(_p(x), _p(weight), _DT[weight.dtype], _p(shift), _p(scale), ms, _p(out), b, t, c,
                           float(eps), _DT[x.dtype])
    return out


def final_bwd(grad_out: torch.Tensor, x: torch.Tensor, weight: torch.Tensor, scale: torch.Tensor, eps: float):
    """Autograd of final_fwd: (grad_x, grad_weight fp32 [C], grad_shift fp32 [B,C], grad_scale fp32 [B,C])."""
    x, weight, gm = _c(x), _c(weight), _c(grad_out.to(x.dtype))
    scale = _c(scale)
    b, t, c = x.shape
    gx = torch.empty_like(x)
    gw = torch.empty(c, dtype=torch.float32)
    gsh = torch.empty(b, c, dtype=torch.float32)
    gsc = torch.empty(b, c, dtype=torch.float32)
    lib().oracle_final_bwd(_p(x), _p(weight), _DT[weight.dtype], _p(scale), c, _p(gm), _p(gx), _p(gw), _p(gsh),
                           _p(gsc), b, t, c, float(eps), _DT[x.dtype])
    return gx, gw, gsh, gsc


def branch_fwd(z, dz_attn, mlp_out, gate, alpha, beta):
    """WorkspaceSharedAdaLNBranch's output sum (local_thc.py:318-323) then the lazy
    update (:1325-1328): (dz, z').  z, dz_attn, mlp_out [B,T,C]; gate [B,C]."""
    z, dz_attn, mlp_out, gate, alpha, beta = (_c(t) for t in (z, dz_attn, mlp_out, gate, alpha, beta))
    b, t, c = z.shape
    dz, zo = torch.empty_like(z), torch.empty_like(z)
    lib().oracle_branch_fwd(_p(z), _p(dz_attn), _p(mlp_out), _p(gate), c, _p(alpha), _DT[alpha.dtype], _p(beta),
                            _DT[beta.dtype], _p(dz), _p(zo), b, t, c, _DT[z.dtype])
    return dz, zo


def branch_bwd(g_dz, g_zo, dz, mlp_out, gate, alpha, beta):
    """Autograd of branch_fwd: (grad dz_attn, grad mlp_out, grad gate fp32 [B,C],
    grad alpha fp32, grad beta fp32); g_dz may be None."""
    g_zo, dz, mlp_out, gate, alpha, beta = (_c(t) for t in (g_zo, dz, mlp_out, gate, alpha, beta))
    g_dz = _c(g_dz) if g_dz is not None else None
    b, t, c = dz.shape
    g_attn, g_mlp = torch.empty_like(dz), torch.empty_like(dz)
    g_gate = torch.empty(b, c, dtype=torch.float32)
    ga, gb = torch.empty(c, 16, dtype=torch.float32), torch.empty(c, 16, dtype=torch.float32)
    lib().oracle_branch_bwd(_p(g_dz), _p(g_zo), _p(dz), _p(mlp_out), _p(gate), c, _p(alpha), _DT[alpha.dtype],
                            _p(beta), _DT[beta.dtype], _p(g_attn), _p(g_mlp), _p(g_gate), _p(ga), _p(gb), b, t, c,
                            _DT[dz.dtype])
    return g_attn, g_mlp, g_gate, ga, gb


__all__ = ["lib", "num_threads", "set_num_threads", "read", "write", "write_add", "materialise", "materialise_bwd",
           "weight_grad", "lazy_fwd", "lazy_bwd", "final_fwd", "final_bwd", "branch_fwd", "branch_bwd", "OUT"]
