"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations of the LTHC interface.

  config 1: read + write, fp32, X[B=2, 256 cells, 16 pos, C=768] ~ N(0,1),
            read weights R[C,16] ~ N(1/16, 0.01) (used directly as alpha),
            write weights P[C,16] ~ N(0, 0.02), dZ[2,256,C] ~ N(0,1), seed 0
  config 2: fused materialisation, bf16, X_0[64,256,16,768] ~ N(0,1),
            dZ[12,64,256,768] ~ N(0, 0.1), P_l[12,768,16] ~ N(0, 0.02) fp32

X is generated cell-major [B, G*G, 16, C] and laid out as the NHWC residual
[B, 4G, 4G, C] the model uses (cell (wy, wx), position r = 4*row + col).
Generation runs on the target device with a seeded torch.Generator so the GPU
benchmark does not pay for host-side random numbers.
"""
from __future__ import annotations

import torch


def cell_major_to_nhwc(x: torch.Tensor) -> torch.Tensor:
    """[B, G*G, 16, C] -> [B, 4G, 4G, C]."""
    b, n, r, c = x.shape
    g = int(round(n ** 0.5))
    if g * g != n or r != 16:
        raise ValueError(f"expected [B, G*G, 16, C], got {tuple(x.shape)}")
    return x.view(b, g, g, 4, 4, c).permute(0, 1, 3, 2, 4, 5).reshape(b, 4 * g, 4 * g, c).contiguous()


def nhwc_to_cell_major(x: torch.Tensor) -> torch.Tensor:
    """[B, 4G, 4G, C] -> [B, G*G, 16, C]."""
    b, h, w, c = x.shape
    g = h // 4
    return x.view(b, g, 4, g, 4, c).permute(0, 1, 3, 2, 4, 5).reshape(b, g * g, 16, c).contiguous()


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _randn(shape, gen, device, dtype, mean=0.0, std=1.0, chunk_elems: int = 1 << 26) -> torch.Tensor:
    """N(mean, std) in `dtype`, drawn in fp32 chunks to bound the temporary memory."""
    out = torch.empty(shape, device=device, dtype=dtype)
    flat = out.view(-1)
    for s in range(0, flat.numel(), chunk_elems):
        n = min(chunk_elems, flat.numel() - s)
        t = torch.randn(n, generator=gen, device=device, dtype=torch.float32)
        if std != 1.0:
            t.mul_(std)
        if mean != 0.0:
            t.add_(mean)
        flat[s:s + n].copy_(t)
    return out


def residual(B: int, G: int, C: int, *, seed: int, device="cpu", dtype=torch.float32, std: float = 1.0) -> torch.Tensor:
    """X ~ N(0, std^2) as an NHWC residual [B, 4G, 4G, C] (generated cell-major)."""
    gen = _gen(device, seed)
    return cell_major_to_nhwc(_randn((B, G * G, 16, C), gen, device, dtype, std=std))


def config1(*, B: int = 2, G: int = 16, C: int = 768, seed: int = 0, device="cpu", dtype=torch.float32) -> dict:
    gen = _gen(device, seed)
    x = cell_major_to_nhwc(_randn((B, G * G, 16, C), gen, device, dtype))
    R = _randn((C, 16), gen, device, torch.float32, mean=1.0 / 16, std=0.01)
    P = _randn((C, 16), gen, device, torch.float32, std=0.02)
    dz = _randn((B, G * G, C), gen, device, dtype)
    return {"x": x, "R": R, "P": P, "dz": dz, "B": B, "G": G, "C": C}


def config2(*, B: int = 64, G: int = 16, C: int = 768, L: int = 12, seed: int = 0, device="cpu",
            dtype=torch.bfloat16) -> dict:
    gen = _gen(device, seed)
    x0 = cell_major_to_nhwc(_randn((B, G * G, 16, C), gen, device, dtype))
    dz = [_randn((B, G * G, C), gen, device, dtype, std=0.1) for _ in range(L)]
    P = [_randn((C, 16), gen, device, torch.float32, std=0.02) for _ in range(L)]
    R = _randn((C, 16), gen, device, torch.float32, mean=1.0 / 16, std=0.01)
    return {"x0": x0, "dz": dz, "P": P, "R": R, "B": B, "G": G, "C": C, "L": L}


def materialise_bytes(B: int, G: int, C: int, L: int, act_bytes: int, w_bytes: int = 4, has_x0: bool = True) -> int:
    """Algorithmic HBM bytes of one materialisation: read X_0 and the L updates and
    weights, write X_L once (1,107,886,080 B at config 2)."""
    hi = B * 16 * G * G * C
    lo = B * G * G * C
    return (hi * (2 if has_x0 else 1) + L * lo) * act_bytes + L * C * 16 * w_bytes


def materialise_bwd_bytes(B: int, G: int, C: int, L: int, act_bytes: int, w_bytes: int = 4) -> int:
    """Read grad_out and the L updates, write the L update grads, read the weights,
    write the fp32 weight grads (1,007,812,608 B at config 2; grad X_0 aliases grad_out)."""
    hi = B * 16 * G * G * C
    lo = B * G * G * C
    return hi * act_bytes + 2 * L * lo * act_bytes + L * C * 16 * (w_bytes + 4)


def materialise_grad_dz_bytes(B: int, G: int, C: int, L: int, act_bytes: int, w_bytes: int = 4) -> int:
    """The backward's pooling half alone: read grad_out and the weights, write the L update grads."""
    return (B * 16 * G * G * C + L * B * G * G * C) * act_bytes + L * C * 16 * w_bytes


def materialise_grad_beta_bytes(B: int, G: int, C: int, L: int, act_bytes: int) -> int:
    """The backward's weight-gradient half alone: read grad_out and the L updates, write the fp32 weight grads."""
    return (B * 16 * G * G * C + L * B * G * G * C) * act_bytes + L * C * 16 * 4


def read_bytes(B: int, G: int, C: int, act_bytes: int, w_bytes: int) -> int:
    hi = B * 16 * G * G * C
    lo = B * G * G * C
    return (hi + lo) * act_bytes + C * 16 * w_bytes


def write_add_bytes(B: int, G: int, C: int, act_bytes: int, w_bytes: int) -> int:
    hi = B * 16 * G * G * C
    lo = B * G * G * C
    return (2 * hi + lo) * act_bytes + C * 16 * w_bytes


def read_bwd_bytes(B: int, G: int, C: int, act_bytes: int, w_bytes: int) -> int:
    """grad_x = alpha (.) grad_z and grad_alpha = sum x*grad_z in one pass: read x and
    grad_z once, write grad_x and the fp32 [C,16] gradient."""
    hi = B * 16 * G * G * C
    lo = B * G * G * C
    return (2 * hi + lo) * act_bytes + C * 16 * (w_bytes + 4)


def lazy_bytes(N: int, C: int, act_bytes: int, w_bytes: int) -> int:
    return 3 * N * C * act_bytes + 2 * C * 16 * w_bytes


def branch_fwd_bytes(N: int, B: int, C: int, act_bytes: int, w_bytes: int) -> int:
    """Branch epilogue + lazy update over N = B*T rows: read z, dz_attn, mlp_out,
    write dz and z' (5 row passes; the reference's four elementwise kernels make
    10), plus the gate rows and the weights."""
    return 5 * N * C * act_bytes + B * C * act_bytes + 2 * C * 16 * w_bytes


def branch_bwd_bytes(N: int, B: int, C: int, act_bytes: int, w_bytes: int) -> int:
    """Its backward: read grad dz, grad z', dz, mlp_out, write grad dz_attn and
    grad mlp_out; gate rows, weights and the fp32 gate / alpha / beta gradients."""
    return 6 * N * C * act_bytes + B * C * (act_bytes + 4) + 2 * C * 16 * (w_bytes + 4)


def final_fwd_bytes(B: int, T: int, C: int, act_bytes: int, w_bytes: int = 4) -> int:
    """Final-layer norm + modulate: read x, write m, read the norm weight and the
    image's shift / scale rows (805,318,656 + ... B at B = 64, T = 4096, C = 768)."""
    return 2 * B * T * C * act_bytes + C * w_bytes + 2 * B * C * act_bytes


def final_bwd_bytes(B: int, T: int, C: int, act_bytes: int, w_bytes: int = 4) -> int:
    """Its backward: read x and grad m, write grad x; weight, scale rows and the
    fp32 weight / shift / scale gradients are small."""
    return 3 * B * T * C * act_bytes + C * w_bytes + B * C * act_bytes + (C + 2 * B * C) * 4


def embed_bytes(B: int, H: int, C: int, in_ch: int = 3, img_bytes: int = 4) -> int:
    """Patch embedding + read: read the images, write X0 [B,H,H,C] and Z [B,(H/4)^2,C]
    in bf16, read the bf16 weights (479,203,072 B at B = 64, H = 64, C = 768)."""
    return (B * in_ch * 16 * H * H * img_bytes + 2 * B * H * H * C + 2 * B * (H // 4) ** 2 * C
            + 2 * (128 * in_ch * 16 + C * 128 + C + 16 * C))


def embed_flops(B: int, H: int, C: int, in_ch: int = 3) -> int:
    """Multiply-adds x 2 of the two convolutions as GEMMs (54.8 GFLOP at B = 64)."""
    return 2 * B * H * H * (in_ch * 16 * 128 + 128 * C)

