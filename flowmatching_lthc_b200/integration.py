"""Drop-in installation of the B200 kernels behind an existing ``flowmatching_lthc``.

    import flowmatching_lthc.models.local_thc            # the user's reference package
    from flowmatching_lthc_b200 import integration
    handle = integration.install()                        # patches the LTHC methods
    model = build_model("lthc_b4_velocity").cuda()        # unchanged API, keys, signatures
    ...
    handle.uninstall()                                    # restores the original methods

Patched methods (``flowmatching_lthc/models/local_thc.py``):

  SharedLocalRead.read                                           :1211-1223
  LayerLocalWrite.write / write_add                              :1261-1276
  SharedReadLocalTHCSharedAdaLNJiTBlock.lazy_workspace_update    :1325-1328
  SharedReadLocalTHCSharedAdaLNJiT.final_accumulate_reference    :1368-1372 (pure-torch loop)
  SharedReadFusedFinalLocalTHCSharedAdaLNJiT.final_accumulate_reference   :1407-1410 (stacked op)
  SharedReadFusedFinal12LocalTHCSharedAdaLNJiT.final_accumulate_reference :1416-1420 (released op)
  FinalLayerSharedAdaLN.forward (RMSNorm + modulate fused; the Linear stays)   :865-873
  SharedReadLocalTHCSharedAdaLNJiT.forward_lazy (patch embedding + shared read
      fused on the tensor cores under bf16 autocast; each block's two AdaLN
      prologues, :320-322, on the norm + modulate kernel and its branch
      epilogue, :318-323, fused with its lazy update)                  :1374-1388

Shape checks and messages are the reference's own; the arithmetic runs in
``liblthc_b200.so``.  The patched methods accept CUDA tensors only (a CPU tensor
raises); call ``uninstall()`` to get the original eager code back.
"""
from __future__ import annotations

import importlib
from dataclasses import dataclass, field
from types import ModuleType

import torch

from . import ops
from .modules import per_channel


def _read(self, x: torch.Tensor) -> torch.Tensor:
    b, h, w, c = x.shape
    hh = self.high_grid
    if h != hh or w != hh or c != self.hidden_size:
        raise ValueError(f"expected [B,{hh},{hh},{self.hidden_size}], got {tuple(x.shape)}")
    return ops.call(ops.read, x, per_channel(self.alpha(dtype=x.dtype), self.hidden_size))


def _check_dz(self, dz: torch.Tensor) -> None:
    b, n, c = dz.shape
    gw = self.workspace_grid
    if n != gw * gw or c != self.hidden_size:
        raise ValueError(f"expected [B,{gw * gw},{self.hidden_size}], got {tuple(dz.shape)}")


def _write(self, dz: torch.Tensor) -> torch.Tensor:
    _check_dz(self, dz)
    return ops.call(ops.write, dz, per_channel(self.beta(dtype=dz.dtype), self.hidden_size))


def _write_add(self, x_hi: torch.Tensor, dz: torch.Tensor) -> torch.Tensor:
    _check_dz(self, dz)
    return ops.call(ops.write_add, x_hi, dz, per_channel(self.beta(dtype=dz.dtype), self.hidden_size))


def _lazy_workspace_update(self, z: torch.Tensor, dz: torch.Tensor, shared_read) -> torch.Tensor:
    alpha = shared_read.alpha(dtype=dz.dtype)
    beta = self.write.beta(dtype=alpha.dtype)
    c = z.shape[-1]
    return ops.call(ops.lazy_update, z, dz, per_channel(alpha, c), per_channel(beta, c))


def _final_loop(self, x0: torch.Tensor, dz_list: list[torch.Tensor]) -> torch.Tensor:
    # the pure-torch loop casts each beta to the update dtype (write_add)
    betas = [per_channel(b.write.beta(dtype=d.dtype), x0.shape[-1]) for b, d in zip(self.blocks, dz_list, strict=True)]
    return ops.call(ops.materialise, x0, list(dz_list), betas)


def _final_stacked(self, x0: torch.Tensor, dz_list: list[torch.Tensor]) -> torch.Tensor:
    betas = [per_channel(b.write.write_weight, x0.shape[-1]) for b in self.blocks]
    if len(dz_list) != len(betas):
        raise ValueError(f"got {len(dz_list)} workspace updates for {len(betas)} blocks")
    return ops.call(ops.materialise, x0, list(dz_list), betas)


def _final12(self, x0: torch.Tensor, dz_list: list[torch.Tensor]) -> torch.Tensor:
    if len(dz_list) != 12 or len(self.blocks) != 12:
        raise ValueError("SharedReadFusedFinal12LocalTHCSharedAdaLNJiT requires depth=12")
    betas = [per_channel(b.write.write_weight, x0.shape[-1]) for b in self.blocks]
    return ops.call(ops.materialise, x0, list(dz_list), betas)


def _final_layer(self, x: torch.Tensor, t2: torch.Tensor) -> torch.Tensor:
    shift, scale = t2.chunk(2, dim=1)
    norm = self.norm_final
    if x.dtype != shift.dtype or x.dim() != 3 or x.shape[-1] > ops.FINAL_MAX_CHANNELS:
        # a dtype mix the fused kernel does not take: the reference's own expression
        return self.linear(_ORIGINAL_MODULATE(norm(x), shift, scale))
    return self.linear(ops.call(ops.final_norm_modulate, x, norm.weight, shift, scale, norm.eps))


_ORIGINAL_MODULATE = None
_LTHC = None  # the patched reference module


def _embed_and_read(model, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """X0 = x_embedder(x) and Z = shared_read.read(X0); one fused tensor-core pass
    under bf16 autocast when the embedder is the bottleneck patch embedding the
    kernel takes, else the two calls."""
    emb, sr = model.x_embedder, model.shared_read
    fused = (x.is_cuda and torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16
             and all(hasattr(emb, a) for a in ("proj1", "proj2", "img_size")) and emb.proj2.bias is not None
             and emb.proj1.bias is None and tuple(x.shape[-2:]) == tuple(emb.img_size)
             and ops.embed_supported(x, emb.proj1.weight, emb.proj2.weight)
             and sr.high_grid == x.shape[-1] // 4 and sr.hidden_size == emb.proj2.weight.shape[0])
    if not fused:
        x0 = emb(x)
        return x0, sr.read(x0)
    c = emb.proj2.weight.shape[0]
    alpha = per_channel(sr.alpha(dtype=torch.bfloat16), c)
    return ops.call(ops.patch_embed_read, x, emb.proj1.weight, emb.proj2.weight, emb.proj2.bias, alpha)


def _norm_modulate(norm, x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """modulate(norm(x), shift, scale) (local_thc.py:320-322) as one norm + modulate
    kernel when norm is the reference's own RMSNorm and x, shift, scale share a
    dtype; otherwise the reference's expression."""
    if (_LTHC is not None and type(norm).forward is _LTHC.RMSNorm.forward and x.is_cuda and x.dim() == 3
            and x.dtype == shift.dtype == scale.dtype and x.shape[-1] % 8 == 0
            and x.shape[-1] <= ops.FINAL_MAX_CHANNELS):
        return ops.call(ops.final_norm_modulate, x, norm.weight, shift, scale, norm.eps)
    return _ORIGINAL_MODULATE(norm(x), shift, scale)


def _branch_and_update(block, z: torch.Tensor, t6: torch.Tensor, rope, shared_read) -> tuple[torch.Tensor, torch.Tensor]:
    """dz = block.branch_update(z, t6, rope) and z' = block.lazy_workspace_update(z, dz,
    shared_read), with the branch's output epilogue (gate product and sum,
    local_thc.py:318-323) and the lazy update as one pass over the rows.  Other
    branch types, overridden methods and dtype mixes take the two calls."""
    br = block.branch
    fused = (_LTHC is not None and type(br).forward is _LTHC.WorkspaceSharedAdaLNBranch.forward
             and type(block).branch_update is _LTHC.SharedReadLocalTHCSharedAdaLNJiTBlock.branch_update
             and type(block).lazy_workspace_update is _lazy_workspace_update and z.is_cuda and z.dim() == 3)
    if not fused:
        dz = block.branch_update(z, t6, rope)
        return dz, block.lazy_workspace_update(z, dz, shared_read)
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = t6.chunk(6, dim=-1)
    dz_attn = gate_msa.unsqueeze(1) * br.attn(_norm_modulate(br.norm1, z, shift_msa, scale_msa), rope)
    mlp_out = br.mlp(_norm_modulate(br.norm2, z + dz_attn, shift_mlp, scale_mlp))
    if not (z.dtype == dz_attn.dtype == mlp_out.dtype == gate_mlp.dtype):
        dz = dz_attn + gate_mlp.unsqueeze(1) * mlp_out
        return dz, block.lazy_workspace_update(z, dz, shared_read)
    alpha = shared_read.alpha(dtype=dz_attn.dtype)
    beta = block.write.beta(dtype=alpha.dtype)
    c = z.shape[-1]
    return ops.call(ops.branch_lazy_update, z, dz_attn, mlp_out, gate_mlp, per_channel(alpha, c), per_channel(beta, c))


def _forward_lazy(self, x: torch.Tensor, t: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    # the reference's lazy forward (local_thc.py:1374-1388) with the patch embedding
    # and the shared read as one call
    cond = self.t_embedder(t) + self.y_embedder(y)
    t6 = self.shared_adaLN_modulation(cond)
    t2 = self.shared_final_modulation(cond)
    x0, z = _embed_and_read(self, x)
    updates = []
    for block in self.blocks:
        dz, z = _branch_and_update(block, z, t6, self.workspace_rope, self.shared_read)
        updates.append(dz)
    x_hi = self.final_accumulate_reference(x0, updates)
    b, hh, wh, c_dim = x_hi.shape
    return self.unpatchify(self.final_layer(x_hi.reshape(b, hh * wh, c_dim), t2))


PATCHES = (
    ("SharedLocalRead", "read", _read),
    ("LayerLocalWrite", "write", _write),
    ("LayerLocalWrite", "write_add", _write_add),
    ("SharedReadLocalTHCSharedAdaLNJiTBlock", "lazy_workspace_update", _lazy_workspace_update),
    ("SharedReadLocalTHCSharedAdaLNJiT", "final_accumulate_reference", _final_loop),
    ("SharedReadFusedFinalLocalTHCSharedAdaLNJiT", "final_accumulate_reference", _final_stacked),
    ("SharedReadFusedFinal12LocalTHCSharedAdaLNJiT", "final_accumulate_reference", _final12),
    ("FinalLayerSharedAdaLN", "forward", _final_layer),
    ("SharedReadLocalTHCSharedAdaLNJiT", "forward_lazy", _forward_lazy),
)


@dataclass
class Installation:
    module: ModuleType
    saved: list = field(default_factory=list)

    def uninstall(self) -> None:
        for cls, name, had, fn in reversed(self.saved):
            if had:
                setattr(cls, name, fn)
            else:
                delattr(cls, name)
        self.saved.clear()

    def __enter__(self) -> "Installation":
        return self

    def __exit__(self, *exc) -> None:
        self.uninstall()


def install(local_thc: ModuleType | None = None) -> Installation:
    """Route the reference model's LTHC methods through the B200 kernels."""
    if local_thc is None:
        local_thc = importlib.import_module("flowmatching_lthc.models.local_thc")
    global _ORIGINAL_MODULATE, _LTHC
    _ORIGINAL_MODULATE = local_thc.modulate
    _LTHC = local_thc
    inst = Installation(local_thc)
    for cls_name, meth, fn in PATCHES:
        cls = getattr(local_thc, cls_name, None)
        if cls is None:
            continue
        had = meth in cls.__dict__
        inst.saved.append((cls, meth, had, cls.__dict__.get(meth)))
        setattr(cls, meth, fn)
    return inst


__all__ = ["install", "Installation", "PATCHES"]
