"""Generates the whole-model golden fixtures (tests/golden/model_*.pt, b4_state_dict_keys.json)
by running the reference's own model and sampler (tongtongliang/flowmatching_lthc) on CPU.

    LTHC_REFERENCE=/path/to/flowmatching_lthc python tests/golden/make_model_golden.py

The reference is needed only here; the GPU tests compare the standalone model of
``flowmatching_lthc_b200.model`` with these files.  Weights are not stored: both
sides fill the same state-dict names with ``model.fill_seeded_`` (values depend
only on the seed and the parameter name), so the fixtures hold inputs, outputs
and gradients only.  Reference code used (paths inside the reference repository):

  SharedReadLocalTHCSharedAdaLNJiT.forward_lazy / forward_naive  flowmatching_lthc/models/local_thc.py:1357-1394
      (the lazy path with the pure-torch materialisation loop, :1368-1372: the
      Triton op of the released subclass does not run on CPU; in fp32 both compute
      X_0 + sum_l P_l(dz_l))
  sample_heun / cfg_velocity (two-call CFG)                      flowmatching_lthc/sampling.py:15-53
  build_model("lthc_b4_velocity") state-dict names and shapes    flowmatching_lthc/models/__init__.py:17-28
  the released LTHC-B/4 size (model_b4): inputs regenerated from the seed, outputs sampled
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
if not os.environ.get("LTHC_REFERENCE"):
    sys.exit("set LTHC_REFERENCE to the root of a flowmatching_lthc checkout (the directory that holds "
             "flowmatching_lthc/models/local_thc.py)")
sys.path.insert(0, os.environ["LTHC_REFERENCE"])
sys.path.insert(0, str(ROOT))
sys.dont_write_bytecode = True

from flowmatching_lthc import sampling as S  # noqa: E402
from flowmatching_lthc.models import build_model as ref_build_model  # noqa: E402
from flowmatching_lthc.models import local_thc as L  # noqa: E402

from flowmatching_lthc_b200.model import fill_seeded_  # noqa: E402

# name -> (model kwargs, batch, weight seed, input seed)
CASES = {
    # 16x16 residual, 4x4 workspace, C = 64: the fp32 parity case (forward, naive, gradients, sampler)
    "model_small": (dict(input_size=64, patch_size=4, hidden_size=64, depth=12, num_heads=4, bottleneck_dim=32,
                         workspace_grid=4, num_classes=10), 2, 3, 4),
    # 32x32 residual, 8x8 workspace, C = 256, bottleneck 128: shapes the tensor-core patch embedding
    # takes, so the bf16 autocast path runs every fused kernel
    "model_wide": (dict(input_size=128, patch_size=4, hidden_size=256, depth=12, num_heads=4, bottleneck_dim=128,
                        workspace_grid=8, num_classes=10), 2, 5, 6),
}
# The released LTHC-B/4 itself (91.6 M parameters) at B = 2: outputs only, a fixed 1-in-7 sample of them.
B4_CASE = ("model_b4", dict(input_size=256, patch_size=4, hidden_size=768, depth=12, num_heads=12, bottleneck_dim=128,
                            workspace_grid=16, num_classes=1000), 2, 7, 8)
B4_SAMPLE_STRIDE = 7
# gradients kept for every case (small tensors) and, in the small case only, the larger ones
GRAD_PARAMS = ("shared_read.read_logits", "blocks.0.write.write_weight", "blocks.11.write.write_weight",
               "final_layer.linear.weight", "final_layer.norm_final.weight", "x_embedder.proj1.weight")
GRAD_PARAMS_SMALL = ("x_embedder.proj2.weight", "blocks.0.branch.attn.qkv.weight", "blocks.5.branch.mlp.w3.weight",
                     "shared_adaLN_modulation.1.weight", "shared_final_modulation.1.weight")


def reference_model(kw: dict, seed: int) -> torch.nn.Module:
    m = L.SharedReadLocalTHCSharedAdaLNJiT(**kw, pool_groups=kw["hidden_size"])
    fill_seeded_(m, seed)
    return m.eval()


def make(name: str) -> dict:
    kw, B, wseed, iseed = CASES[name]
    m = reference_model(kw, wseed)
    gen = torch.Generator().manual_seed(iseed)
    n = kw["input_size"]
    x = torch.randn(B, 3, n, n, generator=gen)
    t = torch.rand(B, generator=gen)
    y = torch.randint(0, kw["num_classes"] + 1, (B,), generator=gen)  # includes the null label
    y[-1] = kw["num_classes"]
    w_out = torch.randn(B, 3, n, n, generator=gen)

    out: dict = {"meta": {"name": name, "kwargs": kw, "batch": B, "weight_seed": wseed, "input_seed": iseed},
                 "x": x, "t": t, "y": y, "w_out": w_out}
    small = name == "model_small"
    with torch.no_grad():
        out["out_naive"] = m(x, t, y, use_lazy=False)
        # the reference's own bf16-autocast output (CPU): how far bf16 arithmetic alone
        # moves the output from the fp32 one, the yardstick of the bf16 GPU checks
        with torch.autocast("cpu", dtype=torch.bfloat16):
            out["out_lazy_bf16_cpu"] = m(x, t, y, use_lazy=True).float()
    with torch.no_grad():
        # interface tensors of the lazy path: X0, Z0, every dz_l and z_l, X_L
        c = m.t_embedder(t) + m.y_embedder(y)
        t6 = m.shared_adaLN_modulation(c)
        x0 = m.x_embedder(x)
        z = m.shared_read.read(x0)
        out["x0"], out["z0"] = x0, z
        dzs, zs = [], []
        for blk in m.blocks:
            dz = blk.branch_update(z, t6, m.workspace_rope)
            z = blk.lazy_workspace_update(z, dz, m.shared_read)
            dzs.append(dz)
            zs.append(z)
        out["dz"], out["z"] = torch.stack(dzs), torch.stack(zs)
        out["x_L"] = m.final_accumulate_reference(x0, dzs)
    if not small:  # keep the committed file small: outputs and small gradients only
        for k in ("x0", "z0", "dz", "z", "x_L"):
            del out[k]
    # forward_lazy with autograd: the output and the gradients of a fixed projection of it
    xg = x.clone().requires_grad_(True)
    o = m(xg, t, y, use_lazy=True)
    out["out_lazy"] = o.detach()
    (o * w_out).sum().backward()
    params = dict(m.named_parameters())
    out["grads"] = {p: params[p].grad.detach().clone() for p in GRAD_PARAMS + (GRAD_PARAMS_SMALL if small else ())}
    out["grad_x"] = xg.grad.detach()

    if small:
        # the reference's two-call CFG Heun sampler, 4 steps, both prediction targets; its
        # noise is the first draw after torch.manual_seed(seed), saved for the doubled-batch sampler
        labels = torch.tensor([3, 7])
        for pred, seed in (("velocity", 21), ("clean", 22)):
            torch.manual_seed(seed)
            noise = torch.randn(2, 3, n, n)
            torch.manual_seed(seed)
            img = S.sample_heun(m, labels, image_size=n, steps=4, cfg_scale=1.5, interval=(0.1, 1.0),
                                num_classes=kw["num_classes"], prediction=pred)
            out[f"sample_{pred}"] = {"labels": labels, "noise": noise, "images": img}
    return out


def make_b4() -> dict:
    name, kw, B, wseed, iseed = B4_CASE
    m = reference_model(kw, wseed)
    gen = torch.Generator().manual_seed(iseed)
    x = torch.randn(B, 3, 256, 256, generator=gen)
    t = torch.rand(B, generator=gen)
    y = torch.tensor([207, kw["num_classes"]])  # a class and the CFG null label
    idx = torch.arange(0, B * 3 * 256 * 256, B4_SAMPLE_STRIDE)
    with torch.no_grad():
        lazy = m(x, t, y, use_lazy=True)
        naive = m(x, t, y, use_lazy=False)
        with torch.autocast("cpu", dtype=torch.bfloat16):
            lazy_bf16 = m(x, t, y, use_lazy=True).float()
    return {"meta": {"name": name, "kwargs": kw, "batch": B, "weight_seed": wseed, "input_seed": iseed,
                     "sample_stride": B4_SAMPLE_STRIDE},
            "t": t, "y": y, "out_lazy_sample": lazy.reshape(-1)[idx].clone(),
            "out_naive_sample": naive.reshape(-1)[idx].clone(),
            "out_lazy_bf16_cpu_sample": lazy_bf16.reshape(-1)[idx].clone(),
            "x_sum": x.double().sum().item()}


def b4_keys() -> dict:
    sd = ref_build_model("lthc_b4_velocity").state_dict()
    return {k: list(v.shape) for k, v in sd.items()}


def main() -> None:
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name in CASES:
        case = make(name)
        path = HERE / f"{name}.pt"
        torch.save(case, path)
        print(f"wrote {path} ({path.stat().st_size} bytes)")
    case = make_b4()
    path = HERE / f"{case['meta']['name']}.pt"
    torch.save(case, path)
    print(f"wrote {path} ({path.stat().st_size} bytes)")
    path = HERE / "b4_state_dict_keys.json"
    path.write_text(json.dumps(b4_keys(), indent=0) + "\n")
    print(f"wrote {path}")


if __name__ == "__main__":
    main()
