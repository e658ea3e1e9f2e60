"""Module-level mirror of the reference's LTHC interface, backed by the B200 kernels.

``SharedLocalRead`` and ``LayerLocalWrite`` keep the constructor arguments,
parameter names/shapes (``read_logits`` / ``write_weight``, i.e. the checkpoint
keys), method names, dtype casts and ValueError messages of
``flowmatching_lthc/models/local_thc.py:1168-1283``; only the arithmetic moves
into ``liblthc_b200.so``.  The kernels implement 4x4 cells (the B/4 geometry);
other cell sizes are rejected at construction.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops

CELL = 4


def _check_geometry(high_grid: int, workspace_grid: int, hidden_size: int, pool_groups: int) -> None:
    if high_grid % workspace_grid != 0:
        raise ValueError(f"high_grid={high_grid} must be divisible by workspace_grid={workspace_grid}")
    if hidden_size % pool_groups != 0:
        raise ValueError(f"hidden_size={hidden_size} must be divisible by pool_groups={pool_groups}")
    if high_grid // workspace_grid != CELL:
        raise ValueError(f"the B200 LTHC kernels implement {CELL}x{CELL} cells; "
                         f"got high_grid/workspace_grid = {high_grid // workspace_grid}")


def per_channel(w: torch.Tensor, hidden_size: int) -> torch.Tensor:
    """Expand group weights [pool_groups, 16] to per-channel [C, 16] (identity when groups == C)."""
    gp = w.shape[0]
    if gp == hidden_size:
        return w
    return w.repeat_interleave(hidden_size // gp, dim=0)


class SharedLocalRead(nn.Module):
    """Depth-shared local read [B,Hh,Hh,C] -> [B,Gw*Gw,C] (local_thc.py:1168-1226)."""

    def __init__(self, high_grid: int, workspace_grid: int, hidden_size: int, pool_groups: int,
                 use_softmax_write: bool = True) -> None:
        super().__init__()
        _check_geometry(high_grid, workspace_grid, hidden_size, pool_groups)
        self.high_grid = high_grid
        self.workspace_grid = workspace_grid
        self.hidden_size = hidden_size
        self.pool_groups = pool_groups
        self.group_dim = hidden_size // pool_groups
        self.cell_size = high_grid // workspace_grid
        self.cell_tokens = self.cell_size * self.cell_size
        self.use_softmax_write = use_softmax_write
        self.read_logits = nn.Parameter(torch.zeros(pool_groups, self.cell_tokens))
        self.reset_parameters()

    def reset_parameters(self) -> None:
        nn.init.constant_(self.read_logits, 0.0)

    def alpha(self, dtype: torch.dtype | None = None) -> torch.Tensor:
        alpha = F.softmax(self.read_logits.float(), dim=-1) if self.use_softmax_write else self.read_logits
        return alpha if dtype is None else alpha.to(dtype=dtype)

    def read(self, x: torch.Tensor) -> torch.Tensor:
        b, h, w, c = x.shape
        hh = self.high_grid
        if h != hh or w != hh or c != self.hidden_size:
            raise ValueError(f"expected [B,{hh},{hh},{self.hidden_size}], got {tuple(x.shape)}")
        return ops.call(ops.read, x, per_channel(self.alpha(dtype=x.dtype), self.hidden_size))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.read(x)


class LayerLocalWrite(nn.Module):
    """Layer-specific local write used with a shared read (local_thc.py:1229-1283)."""

    def __init__(self, high_grid: int, workspace_grid: int, hidden_size: int, pool_groups: int,
                 init_read: float = 1.0) -> None:
        super().__init__()
        _check_geometry(high_grid, workspace_grid, hidden_size, pool_groups)
        self.high_grid = high_grid
        self.workspace_grid = workspace_grid
        self.hidden_size = hidden_size
        self.pool_groups = pool_groups
        self.group_dim = hidden_size // pool_groups
        self.cell_size = high_grid // workspace_grid
        self.cell_tokens = self.cell_size * self.cell_size
        self.write_weight = nn.Parameter(torch.full((pool_groups, self.cell_tokens), float(init_read)))
        self.reset_parameters()

    def reset_parameters(self) -> None:
        nn.init.constant_(self.write_weight, 1.0)

    def beta(self, dtype: torch.dtype | None = None) -> torch.Tensor:
        return self.write_weight if dtype is None else self.write_weight.to(dtype=dtype)

    def _check_dz(self, dz: torch.Tensor) -> None:
        b, n, c = dz.shape
        gw = self.workspace_grid
        if n != gw * gw or c != self.hidden_size:
            raise ValueError(f"expected [B,{gw * gw},{self.hidden_size}], got {tuple(dz.shape)}")

    def write(self, dz: torch.Tensor) -> torch.Tensor:
        self._check_dz(dz)
        return ops.call(ops.write, dz, per_channel(self.beta(dtype=dz.dtype), self.hidden_size))

    def write_add(self, x_hi: torch.Tensor, dz: torch.Tensor) -> torch.Tensor:
        self._check_dz(dz)
        return ops.call(ops.write_add, x_hi, dz, per_channel(self.beta(dtype=dz.dtype), self.hidden_size))

    def gamma_from_alpha(self, alpha: torch.Tensor) -> torch.Tensor:
        beta = self.beta(dtype=alpha.dtype)
        gamma_g = (alpha * beta).sum(dim=-1)
        if self.group_dim == 1:
            return gamma_g
        return gamma_g[:, None].expand(self.pool_groups, self.group_dim).reshape(self.hidden_size)


def lazy_workspace_update(z: torch.Tensor, dz: torch.Tensor, shared_read: SharedLocalRead | nn.Module,
                          write: LayerLocalWrite | nn.Module) -> torch.Tensor:
    """z + gamma_l (.) dz with gamma_l = sum_r alpha*beta_l, one fused kernel
    (SharedReadLocalTHCSharedAdaLNJiTBlock.lazy_workspace_update, local_thc.py:1325-1328)."""
    alpha = shared_read.alpha(dtype=dz.dtype)
    beta = write.beta(dtype=alpha.dtype)
    c = z.shape[-1]
    return ops.call(ops.lazy_update, z, dz, per_channel(alpha, c), per_channel(beta, c))


def final_accumulate(x0: torch.Tensor, dz_list: list[torch.Tensor], writes: list[LayerLocalWrite | nn.Module]) -> torch.Tensor:
    """X_L = X_0 + sum_l P_l(dz_l) in one pass with the fp32 write weights passed
    uncast, as the released model passes them to the Triton op (local_thc.py:1416-1420)."""
    if len(dz_list) != len(writes):
        raise ValueError(f"got {len(dz_list)} workspace updates for {len(writes)} write operators")
    c = x0.shape[-1]
    return ops.call(ops.materialise, x0, list(dz_list), [per_channel(w.write_weight, c) for w in writes])


__all__ = ["SharedLocalRead", "LayerLocalWrite", "lazy_workspace_update", "final_accumulate", "per_channel"]
