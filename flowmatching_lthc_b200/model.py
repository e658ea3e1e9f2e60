"""Standalone LTHC-B/4 flow-matching model whose LTHC interface runs on the B200 kernels.

``build_model("lthc_b4_velocity")`` returns a model with the public API of the
released one (``flowmatching_lthc/models/__init__.py:17-28``): ``model(x, t, y,
use_lazy=None)`` on images ``[B, 3, 256, 256]``, timesteps ``[B]`` and labels
``[B]`` (label ``num_classes`` is the CFG null class), the same constructor
arguments, and a ``state_dict`` whose keys and shapes are those of
``SharedReadFusedFinal12LocalTHCSharedAdaLNJiT`` (``local_thc.py:1413``), so a
checkpoint of the reference loads unchanged (legacy key names are migrated as
``local_thc.py:41-61`` does).  It needs no copy of the reference package.

Every step of the forward that touches the high-resolution residual runs in
``liblthc_b200.so``:

* patch embedding (4x4 conv 3->128, 1x1 conv 128->C) fused with the shared read
  on the tensor cores (bf16 autocast; otherwise the two convolutions and the read
  kernel), ``local_thc.py:84-89, 1378-1379``;
* per block, the branch's output sum ``dz_attn + gate (.) mlp_out`` fused with
  the lazy workspace update ``z + Gamma_l (.) dz`` (``:318-323, 1325-1328``);
* the materialisation ``X_L = X_0 + sum_l P_l(dz_l)`` with the fp32 write
  weights passed uncast (``:1416-1420``);
* the final RMSNorm + shared-AdaLN modulate over the 4096 tokens (``:865-873``).

The same norm + modulate kernel also runs the branch's two AdaLN prologues,
``modulate(norm1(z), shift_msa, scale_msa)`` and ``modulate(norm2(z + dz_attn),
...)`` (``:320-322``): one pass over the workspace rows instead of the eager
chain of casts, reductions and products.

The workspace Transformer between them (RMSNorm, QK-normed attention with 2-D
RoPE through ``scaled_dot_product_attention``, SwiGLU, AdaLN) is plain PyTorch
with the reference's arithmetic (``local_thc.py:175-323``,
``jit_shared_adaln.py:20-60``): it is not LTHC work and stays on library
kernels.  ``forward_naive`` is the literal recurrence (read and write_add per
block, ``:1311-1320, 1357-1366``), the oracle of the lazy identity.
"""
from __future__ import annotations

import math
import re
import zlib

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .modules import LayerLocalWrite, SharedLocalRead, per_channel

MODEL_NAMES = (
    "lthc_b4_velocity",
    "local_thc_jit_shared_read_fused_final12_shared_adaln_b4",
    "local_thc_jit_shared_write_fused_final12_shared_adaln_b4",
)


# ---------------------------------------------------------------------------
# workspace Transformer pieces (library kernels; the reference's arithmetic)
# ---------------------------------------------------------------------------
class RMSNorm(nn.Module):
    """x / rms(x) * weight in fp32, returned in x's dtype (jit_shared_adaln.py:20-30)."""

    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        inv = torch.rsqrt(xf.square().mean(-1, keepdim=True) + self.eps)
        return (xf * inv * self.weight).to(x.dtype)


def modulate(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """Shared-AdaLN modulation of token rows by per-image shift / scale (local_thc.py:37-38)."""
    return x * (1 + scale.unsqueeze(1)) + shift.unsqueeze(1)


def norm_modulate(norm: RMSNorm, x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """modulate(norm(x), shift, scale) over token rows [B, T, C]: one kernel
    (lthc_final_norm_modulate, the reference's op-by-op rounding) when x, shift and
    scale share a dtype, else the eager expression.  The shift / scale halves of a
    chunked AdaLN output are read in place."""
    if (x.is_cuda and x.dim() == 3 and x.dtype == shift.dtype == scale.dtype and x.shape[-1] % 8 == 0
            and x.shape[-1] <= ops.FINAL_MAX_CHANNELS):
        return ops.call(ops.final_norm_modulate, x, norm.weight, shift, scale, norm.eps)
    return modulate(norm(x), shift, scale)


def _rope_tables(half_head_dim: int, grid: int, theta: float = 10000.0) -> tuple[torch.Tensor, torch.Tensor]:
    """cos / sin of the 2-D rotary embedding of a grid x grid workspace
    (jit_shared_adaln.py:40-60): the first half of each head's channels rotates by
    the token's row, the second half by its column, each channel pair (2i, 2i+1)
    by the same angle."""
    inv = 1.0 / theta ** (torch.arange(0, half_head_dim, 2).float()[: half_head_dim // 2] / half_head_dim)
    ang = torch.arange(grid).float()[:, None] * inv[None, :]          # [grid, half/2]
    ang = ang.repeat_interleave(2, dim=-1)                               # [grid, half]
    rows = ang[:, None, :].expand(grid, grid, -1)
    cols = ang[None, :, :].expand(grid, grid, -1)
    table = torch.cat([rows, cols], dim=-1).reshape(grid * grid, -1)    # [grid^2, head_dim]
    return table.cos(), table.sin()


class WorkspaceRope(nn.Module):
    """Applies the 2-D RoPE to [..., tokens, head_dim] (pairs (x0, x1) -> (-x1, x0))."""

    def __init__(self, half_head_dim: int, grid: int) -> None:
        super().__init__()
        cos, sin = _rope_tables(half_head_dim, grid)
        self.register_buffer("freqs_cos", cos, persistent=False)
        self.register_buffer("freqs_sin", sin, persistent=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        pairs = x.unflatten(-1, (-1, 2))
        rot = torch.stack((-pairs[..., 1], pairs[..., 0]), dim=-1).flatten(-2)
        return x * self.freqs_cos.to(x.dtype) + rot * self.freqs_sin.to(x.dtype)


class WorkspaceAttention(nn.Module):
    """Self-attention over the workspace tokens with RMS-normed q / k and 2-D RoPE
    (local_thc.py:207-261)."""

    def __init__(self, dim: int, num_heads: int, attn_drop: float = 0.0, proj_drop: float = 0.0) -> None:
        super().__init__()
        if dim % num_heads:
            raise ValueError(f"dim={dim} must be divisible by num_heads={num_heads}")
        self.num_heads = num_heads
        self.head_dim = dim // num_heads
        self.qkv = nn.Linear(dim, 3 * dim)
        self.q_norm = RMSNorm(self.head_dim)
        self.k_norm = RMSNorm(self.head_dim)
        self.proj = nn.Linear(dim, dim)
        self.attn_drop = attn_drop
        self.proj_drop = proj_drop

    def forward(self, x: torch.Tensor, rope: WorkspaceRope) -> torch.Tensor:
        b, n, c = x.shape
        q, k, v = self.qkv(x).view(b, n, 3, self.num_heads, self.head_dim).permute(2, 0, 3, 1, 4).unbind(0)
        q, k = rope(self.q_norm(q)), rope(self.k_norm(k))
        o = F.scaled_dot_product_attention(q, k, v, dropout_p=self.attn_drop if self.training else 0.0)
        o = self.proj(o.transpose(1, 2).reshape(b, n, c))
        return F.dropout(o, self.proj_drop, self.training) if self.proj_drop else o


class SwiGLU(nn.Module):
    """w3(silu(a) * b) with [a, b] = w12(x); hidden width 2/3 of the nominal one (local_thc.py:264-275)."""

    def __init__(self, dim: int, hidden: int, drop: float = 0.0) -> None:
        super().__init__()
        hidden = int(hidden * 2 / 3)
        self.w12 = nn.Linear(dim, 2 * hidden)
        self.w3 = nn.Linear(hidden, dim)
        self.drop = drop

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        a, b = self.w12(x).chunk(2, dim=-1)
        h = F.silu(a) * b
        return self.w3(F.dropout(h, self.drop, self.training) if self.drop else h)


class WorkspaceBranch(nn.Module):
    """The per-block workspace branch with shared AdaLN (local_thc.py:296-323).

    ``parts`` returns (dz_attn, mlp_out, gate_mlp) so that the output sum
    dz_attn + gate_mlp (.) mlp_out can be fused with the lazy update;
    ``forward`` returns the sum itself."""

    def __init__(self, hidden: int, num_heads: int, mlp_ratio: float, attn_drop: float, proj_drop: float) -> None:
        super().__init__()
        self.norm1 = RMSNorm(hidden)
        self.attn = WorkspaceAttention(hidden, num_heads, attn_drop, proj_drop)
        self.norm2 = RMSNorm(hidden)
        self.mlp = SwiGLU(hidden, int(hidden * mlp_ratio), proj_drop)

    def parts(self, z: torch.Tensor, t6: torch.Tensor, rope: WorkspaceRope):
        sh_a, sc_a, g_a, sh_m, sc_m, g_m = t6.chunk(6, dim=-1)
        dz_attn = g_a.unsqueeze(1) * self.attn(norm_modulate(self.norm1, z, sh_a, sc_a), rope)
        mlp_out = self.mlp(norm_modulate(self.norm2, z + dz_attn, sh_m, sc_m))
        return dz_attn, mlp_out, g_m

    def forward(self, z: torch.Tensor, t6: torch.Tensor, rope: WorkspaceRope) -> torch.Tensor:
        dz_attn, mlp_out, g_m = self.parts(z, t6, rope)
        return dz_attn + g_m.unsqueeze(1) * mlp_out


class Block(nn.Module):
    """One LTHC block: its layer-specific write P_l and its workspace branch."""

    def __init__(self, hidden: int, num_heads: int, high_grid: int, workspace_grid: int, pool_groups: int,
                 mlp_ratio: float, attn_drop: float, proj_drop: float) -> None:
        super().__init__()
        self.write = LayerLocalWrite(high_grid, workspace_grid, hidden, pool_groups)
        self.branch = WorkspaceBranch(hidden, num_heads, mlp_ratio, attn_drop, proj_drop)

    @property
    def read(self) -> LayerLocalWrite:
        """Alias of ``write`` kept by the reference for old research checkpoints (local_thc.py:1306-1309)."""
        return self.write

    def branch_update(self, z: torch.Tensor, t6: torch.Tensor, rope: WorkspaceRope) -> torch.Tensor:
        return self.branch(z, t6, rope)

    def lazy_workspace_update(self, z: torch.Tensor, dz: torch.Tensor, shared_read: SharedLocalRead) -> torch.Tensor:
        alpha = shared_read.alpha(dtype=dz.dtype)
        beta = self.write.beta(dtype=alpha.dtype)
        c = z.shape[-1]
        return ops.call(ops.lazy_update, z, dz, per_channel(alpha, c), per_channel(beta, c))

    def branch_and_update(self, z: torch.Tensor, t6: torch.Tensor, rope: WorkspaceRope,
                          shared_read: SharedLocalRead) -> tuple[torch.Tensor, torch.Tensor]:
        """(dz, z_next) with the branch's output sum and the lazy update in one kernel."""
        dz_attn, mlp_out, gate = self.branch.parts(z, t6, rope)
        if not (z.dtype == dz_attn.dtype == mlp_out.dtype == gate.dtype):
            dz = dz_attn + gate.unsqueeze(1) * mlp_out
            return dz, self.lazy_workspace_update(z, dz, shared_read)
        alpha = shared_read.alpha(dtype=dz_attn.dtype)
        beta = self.write.beta(dtype=alpha.dtype)
        c = z.shape[-1]
        return ops.call(ops.branch_lazy_update, z, dz_attn, mlp_out, gate, per_channel(alpha, c), per_channel(beta, c))

    def forward_naive(self, x_hi: torch.Tensor, t6: torch.Tensor, rope: WorkspaceRope,
                      shared_read: SharedLocalRead) -> torch.Tensor:
        return self.write.write_add(x_hi, self.branch(shared_read.read(x_hi), t6, rope))


class TimestepEmbedder(nn.Module):
    """Sinusoidal features of t (cos half, then sin half) through a 2-layer SiLU MLP (local_thc.py:175-196)."""

    def __init__(self, hidden: int, freq_dim: int = 256) -> None:
        super().__init__()
        self.frequency_embedding_size = freq_dim
        self.mlp = nn.Sequential(nn.Linear(freq_dim, hidden), nn.SiLU(), nn.Linear(hidden, hidden))

    @staticmethod
    def timestep_embedding(t: torch.Tensor, dim: int, max_period: int = 10000) -> torch.Tensor:
        half = dim // 2
        freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
        ang = t.float()[:, None] * freqs[None, :]
        emb = torch.cat([ang.cos(), ang.sin()], dim=-1)
        return F.pad(emb, (0, 1)) if dim % 2 else emb

    def forward(self, t: torch.Tensor) -> torch.Tensor:
        return self.mlp(self.timestep_embedding(t, self.frequency_embedding_size))


class LabelEmbedder(nn.Module):
    """Class embedding with one extra row for the CFG null label (local_thc.py:199-205)."""

    def __init__(self, num_classes: int, hidden: int) -> None:
        super().__init__()
        self.num_classes = num_classes
        self.embedding_table = nn.Embedding(num_classes + 1, hidden)

    def forward(self, labels: torch.Tensor) -> torch.Tensor:
        return self.embedding_table(labels)


class PatchEmbed(nn.Module):
    """Bottleneck patch embedding to NHWC tokens: 4x4 conv in->128, 1x1 conv 128->C (local_thc.py:64-89)."""

    def __init__(self, img_size: int, patch_size: int, in_chans: int, bottleneck: int, embed_dim: int) -> None:
        super().__init__()
        self.img_size = (img_size, img_size)
        self.patch_size = (patch_size, patch_size)
        self.proj1 = nn.Conv2d(in_chans, bottleneck, kernel_size=patch_size, stride=patch_size, bias=False)
        self.proj2 = nn.Conv2d(bottleneck, embed_dim, kernel_size=1)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if tuple(x.shape[-2:]) != self.img_size:
            raise ValueError(f"expected image size {self.img_size}, got {tuple(x.shape[-2:])}")
        return self.proj2(self.proj1(x)).permute(0, 2, 3, 1).contiguous()


class FinalLayer(nn.Module):
    """RMSNorm + shared-AdaLN modulate (one kernel) and the Linear to patch pixels (local_thc.py:865-873)."""

    def __init__(self, hidden: int, patch_size: int, out_channels: int) -> None:
        super().__init__()
        self.norm_final = RMSNorm(hidden)
        self.linear = nn.Linear(hidden, patch_size * patch_size * out_channels)

    def forward(self, x: torch.Tensor, t2: torch.Tensor) -> torch.Tensor:
        shift, scale = t2.chunk(2, dim=1)
        return self.linear(norm_modulate(self.norm_final, x, shift, scale))


# ---------------------------------------------------------------------------
# the model
# ---------------------------------------------------------------------------
def migrate_state_dict_keys(state_dict: dict) -> dict:
    """Rename the research checkpoints' swapped read/write keys to the public names
    (the mapping of local_thc.py:41-61: residual->workspace is "read"/read_logits,
    workspace->residual is "write"/write_weight)."""
    rules = ((r"shared_write\.", "shared_read."), (r"blocks\.(\d+)\.read\.", r"blocks.\1.write."),
             (r"\.hyper\.write_logits", ".hyper.read_logits"), (r"\.hyper\.read_weight", ".hyper.write_weight"),
             (r"\.write_logits", ".read_logits"), (r"\.read_weight", ".write_weight"))
    out = {}
    for key, value in state_dict.items():
        for pat, rep in rules:
            key = re.sub(pat, rep, key)
        out[key] = value
    return out


class LTHCModel(nn.Module):
    """Shared-read lazy LTHC flow-matching model (the released LTHC-B/4 at the defaults
    of ``build_model``), constructor arguments as ``LocalTHCJiT`` (local_thc.py:876-895)."""

    def __init__(self, input_size: int = 256, patch_size: int = 4, in_channels: int = 3, hidden_size: int = 768,
                 depth: int = 12, num_heads: int = 12, mlp_ratio: float = 4.0, attn_drop: float = 0.0,
                 proj_drop: float = 0.0, num_classes: int = 1000, bottleneck_dim: int = 128,
                 workspace_grid: int = 16, pool_groups: int | None = None, attn_backend: str = "flash",
                 use_lazy: bool = True) -> None:
        super().__init__()
        high_grid = input_size // patch_size
        if high_grid % workspace_grid:
            raise ValueError(f"input_size/patch_size={high_grid} must be divisible by workspace_grid={workspace_grid}")
        self.input_size, self.patch_size = input_size, patch_size
        self.in_channels = self.out_channels = in_channels
        self.hidden_size, self.depth, self.num_heads = hidden_size, depth, num_heads
        self.num_classes, self.workspace_grid, self.high_grid = num_classes, workspace_grid, high_grid
        self.pool_groups = hidden_size if pool_groups is None else pool_groups
        self.attn_backend = attn_backend
        self.use_lazy = bool(use_lazy)

        self.t_embedder = TimestepEmbedder(hidden_size)
        self.y_embedder = LabelEmbedder(num_classes, hidden_size)
        self.x_embedder = PatchEmbed(input_size, patch_size, in_channels, bottleneck_dim, hidden_size)
        self.workspace_rope = WorkspaceRope(hidden_size // num_heads // 2, workspace_grid)
        # dropout only in the middle half of the blocks, as the reference builds them (local_thc.py:921-931)
        mid = range(depth // 4, depth // 4 * 3)
        self.blocks = nn.ModuleList(
            Block(hidden_size, num_heads, high_grid, workspace_grid, self.pool_groups, mlp_ratio,
                  attn_drop if i in mid else 0.0, proj_drop if i in mid else 0.0) for i in range(depth))
        self.final_layer = FinalLayer(hidden_size, patch_size, self.out_channels)
        self.shared_adaLN_modulation = nn.Sequential(nn.SiLU(), nn.Linear(hidden_size, 6 * hidden_size))
        self.shared_final_modulation = nn.Sequential(nn.SiLU(), nn.Linear(hidden_size, 2 * hidden_size))
        self.shared_read = SharedLocalRead(high_grid, workspace_grid, hidden_size, self.pool_groups)
        self.initialize_weights()

    # -- parameters ---------------------------------------------------------
    def initialize_weights(self) -> None:
        """The reference's initialisation (local_thc.py:945-970, 1000-1007): Xavier-uniform
        Linear and conv weights with zero biases, N(0, 0.02) label table and timestep
        MLP, zero AdaLN heads and final Linear, read logits 0, write weights 1."""
        for mod in self.modules():
            if isinstance(mod, nn.Linear):
                nn.init.xavier_uniform_(mod.weight)
                nn.init.zeros_(mod.bias)
        for conv in (self.x_embedder.proj1, self.x_embedder.proj2):
            nn.init.xavier_uniform_(conv.weight.data.view(conv.weight.shape[0], -1))
        nn.init.zeros_(self.x_embedder.proj2.bias)
        nn.init.normal_(self.y_embedder.embedding_table.weight, std=0.02)
        nn.init.normal_(self.t_embedder.mlp[0].weight, std=0.02)
        nn.init.normal_(self.t_embedder.mlp[2].weight, std=0.02)
        for lin in (self.final_layer.linear, self.shared_adaLN_modulation[-1], self.shared_final_modulation[-1]):
            nn.init.zeros_(lin.weight)
            nn.init.zeros_(lin.bias)

    def load_state_dict(self, state_dict, strict: bool = True, assign: bool = False):
        return super().load_state_dict(migrate_state_dict_keys(state_dict), strict=strict, assign=assign)

    @property
    def shared_write(self) -> SharedLocalRead:
        """Alias of ``shared_read`` kept by the reference for old research code (local_thc.py:1352-1355)."""
        return self.shared_read

    # -- forward ------------------------------------------------------------
    def unpatchify(self, x: torch.Tensor) -> torch.Tensor:
        """[B, h*w, p*p*c] token rows -> [B, c, h*p, w*p] images (local_thc.py:972-980)."""
        b, n, _ = x.shape
        h = math.isqrt(n)
        if h * h != n:
            raise ValueError(f"token count {n} is not square")
        p, c = self.patch_size, self.out_channels
        return x.view(b, h, h, p, p, c).permute(0, 5, 1, 3, 2, 4).reshape(b, c, h * p, h * p)

    def _conditioning(self, t: torch.Tensor, y: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        cond = self.t_embedder(t) + self.y_embedder(y)
        return self.shared_adaLN_modulation(cond), self.shared_final_modulation(cond)

    def _embed_and_read(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """(X0, Z0): one tensor-core pass under bf16 autocast when the kernel takes the
        shapes, else the patch embedding and the read kernel."""
        emb, sr = self.x_embedder, self.shared_read
        if (x.is_cuda and torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16
                and tuple(x.shape[-2:]) == emb.img_size and self.patch_size == 4
                and ops.embed_supported(x, emb.proj1.weight, emb.proj2.weight)):
            alpha = per_channel(sr.alpha(dtype=torch.bfloat16), self.hidden_size)
            return ops.call(ops.patch_embed_read, x, emb.proj1.weight, emb.proj2.weight, emb.proj2.bias, alpha)
        x0 = emb(x)
        return x0, sr.read(x0)

    def final_accumulate_reference(self, x0: torch.Tensor, dz_list: list[torch.Tensor]) -> torch.Tensor:
        """X_L = X_0 + sum_l P_l(dz_l), one kernel, fp32 write weights uncast (local_thc.py:1416-1420)."""
        if len(dz_list) != len(self.blocks):
            raise ValueError(f"got {len(dz_list)} workspace updates for {len(self.blocks)} blocks")
        c = x0.shape[-1]
        betas = [per_channel(b.write.write_weight, c) for b in self.blocks]
        return ops.call(ops.materialise, x0, list(dz_list), betas)

    def _head(self, x_hi: torch.Tensor, t2: torch.Tensor) -> torch.Tensor:
        b, h, w, c = x_hi.shape
        return self.unpatchify(self.final_layer(x_hi.reshape(b, h * w, c), t2))

    def forward_lazy(self, x: torch.Tensor, t: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        t6, t2 = self._conditioning(t, y)
        x0, z = self._embed_and_read(x)
        updates = []
        for block in self.blocks:
            dz, z = block.branch_and_update(z, t6, self.workspace_rope, self.shared_read)
            updates.append(dz)
        return self._head(self.final_accumulate_reference(x0, updates), t2)

    def forward_naive(self, x: torch.Tensor, t: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        t6, t2 = self._conditioning(t, y)
        x_hi = self.x_embedder(x)
        for block in self.blocks:
            x_hi = block.forward_naive(x_hi, t6, self.workspace_rope, self.shared_read)
        return self._head(x_hi, t2)

    def forward(self, x: torch.Tensor, t: torch.Tensor, y: torch.Tensor, use_lazy: bool | None = None) -> torch.Tensor:
        lazy = self.use_lazy if use_lazy is None else use_lazy
        return self.forward_lazy(x, t, y) if lazy else self.forward_naive(x, t, y)


# the class name the reference registry returns for "lthc_b4_velocity"
SharedReadFusedFinal12LocalTHCSharedAdaLNJiT = LTHCModel


def build_model(name: str = "lthc_b4_velocity", **kwargs) -> LTHCModel:
    """The released LTHC-B/4 (patch 4, hidden 768, depth 12, 12 heads, bottleneck 128,
    16x16 workspace, per-channel read/write weights) under its public and research
    names (flowmatching_lthc/models/__init__.py:17-28); kwargs override the defaults."""
    if name not in MODEL_NAMES:
        raise ValueError(f"unknown model: {name}; available={MODEL_NAMES}")
    cfg = dict(patch_size=4, hidden_size=768, depth=12, num_heads=12, bottleneck_dim=128, workspace_grid=16,
               pool_groups=768)
    cfg.update(kwargs)
    return LTHCModel(**cfg)


def fill_seeded_(module: nn.Module, seed: int) -> nn.Module:
    """Overwrite every parameter with seeded CPU random values that keep activations
    O(1) through the network (weights ~ N(0, 1/fan_in), biases ~ N(0, 0.02^2),
    norm weights ~ 1 + N(0, 0.1^2), read logits ~ N(0, 1), write weights
    ~ 1 + N(0, 0.1^2)).  Each parameter's values depend only on the seed and its
    state-dict name, so any module with the reference's keys (this model or the
    reference's own) receives identical weights: the parity fixtures rely on it.
    The zero-initialised AdaLN heads and final Linear of a fresh model would make
    every output zero; this fills them too."""
    with torch.no_grad():
        for name, p in module.named_parameters():
            g = torch.Generator().manual_seed(seed * 1_000_003 + zlib.crc32(name.encode()))
            r = torch.randn(p.shape, generator=g, dtype=torch.float32)
            if name.endswith("read_logits"):
                v = r
            elif name.endswith(("write_weight", "norm.weight", "norm1.weight", "norm2.weight", "norm_final.weight",
                                "q_norm.weight", "k_norm.weight")):
                v = 1.0 + 0.1 * r
            elif name.endswith("bias") or p.dim() == 1:
                v = 0.02 * r
            elif name.endswith("embedding_table.weight"):
                v = r
            else:
                fan_in = p[0].numel()
                v = r / math.sqrt(fan_in)
            p.copy_(v.to(p.dtype))
    return module


__all__ = ["LTHCModel", "SharedReadFusedFinal12LocalTHCSharedAdaLNJiT", "build_model", "MODEL_NAMES",
           "migrate_state_dict_keys", "fill_seeded_", "RMSNorm", "modulate", "WorkspaceRope"]
