"""Heun / classifier-free-guidance sampler with a doubled batch, eager or as one CUDA graph.

Same mathematics and signature as the reference's ``sample_heun`` /
``cfg_velocity`` (``flowmatching_lthc/sampling.py:15-53``): ``steps - 1`` Heun
steps and a final Euler step over ``linspace(0, 1, steps + 1)``, CFG applied
inside ``interval`` with ``v = v_uncond + s * (v_cond - v_uncond)``, and the
"clean" or "velocity" prediction targets.  The difference is the model call:
the reference evaluates the conditional and the unconditional branch as two
separate forward passes of batch B (``sampling.py:16-18``); this sampler
concatenates ``[cond; uncond]`` into one forward pass of batch 2B, which halves
the number of launches per step.  Per sample the arithmetic is the same; with
bf16 GEMMs the rounding can differ slightly with the batch size.

``noise`` may be passed explicitly so that sharded runs reproduce a single-GPU
run; ``image_noise`` draws it per image from a host seed, so that a rank draws
only the images of its own shard and every image gets the same noise whatever
the number of ranks.  ``GraphedHeunSampler`` captures the whole loop (every step,
every model call) for a fixed batch into one CUDA graph, so a sampling run is a
copy in, one graph launch and a copy out: no per-step host dispatch.
"""
from __future__ import annotations

import contextlib

import torch


def _to_velocity(pred, z, t, prediction: str, t_eps: float):
    if prediction == "clean":
        return (pred - z) / (1.0 - t).clamp_min(t_eps)
    if prediction == "velocity":
        return pred
    raise ValueError(f"unknown prediction target: {prediction}")


@torch.no_grad()
def cfg_velocity_doubled(model, z, t, labels, *, num_classes, cfg_scale=1.0, interval=(0.0, 1.0), t_eps=5e-2,
                         prediction="clean"):
    """v_uncond + s (v_cond - v_uncond) from one forward pass on [cond; uncond]."""
    b = z.shape[0]
    null_labels = torch.full_like(labels, num_classes)
    zz = torch.cat([z, z], 0)
    tt = torch.cat([t, t], 0)
    pred = model(zz, tt.flatten(), torch.cat([labels, null_labels], 0))
    v = _to_velocity(pred, zz, tt, prediction, t_eps)
    v_cond, v_uncond = v[:b], v[b:]
    low, high = interval
    mask = (t < high) & ((low == 0) | (t > low))
    scale = torch.where(mask, torch.full_like(t, cfg_scale), torch.ones_like(t))
    return v_uncond + scale * (v_cond - v_uncond)


def _time_grid(steps: int, device) -> list[float]:
    # the reference's grid: float32 linspace on the sampling device, read back per step
    return torch.linspace(0.0, 1.0, steps + 1, device=device).tolist()


def _heun_loop(model, z, labels, ts: list[float], kw: dict):
    """The reference's update sequence (sampling.py:38-53) from state z; no host reads."""
    bsz, device = z.shape[0], z.device
    for i in range(len(ts) - 2):
        t = torch.full((bsz, 1, 1, 1), float(ts[i]), device=device)
        t_next = torch.full((bsz, 1, 1, 1), float(ts[i + 1]), device=device)
        v = cfg_velocity_doubled(model, z, t, labels, **kw)
        z_euler = z + (t_next - t) * v
        v_next = cfg_velocity_doubled(model, z_euler, t_next, labels, **kw)
        z = z + (t_next - t) * 0.5 * (v + v_next)
    t = torch.full((bsz, 1, 1, 1), float(ts[-2]), device=device)
    t_next = torch.full((bsz, 1, 1, 1), float(ts[-1]), device=device)
    v = cfg_velocity_doubled(model, z, t, labels, **kw)
    return z + (t_next - t) * v


@torch.no_grad()
def sample_heun(model, labels, *, image_size=256, noise_scale=1.0, steps=50, cfg_scale=1.0, interval=(0.0, 1.0),
                num_classes=1000, t_eps=5e-2, prediction="clean", noise: torch.Tensor | None = None):
    """Heun sampler of the reference (``sampling.py:26-53``) with doubled-batch CFG."""
    bsz = labels.numel()
    device = labels.device
    if noise is None:
        z = torch.randn(bsz, 3, image_size, image_size, device=device) * noise_scale
    else:
        z = noise.to(device=device, dtype=torch.float32) * noise_scale
    kw = dict(num_classes=num_classes, cfg_scale=cfg_scale, interval=interval, t_eps=t_eps, prediction=prediction)
    return _heun_loop(model, z, labels, _time_grid(steps, device), kw)


def image_noise(seed: int, start: int, stop: int, image_size: int = 256, channels: int = 3) -> torch.Tensor:
    """N(0, 1) noise of images [start, stop) of a run seeded with `seed`, on the host:
    image i draws from its own generator (seed, i), so a shard draws only its images
    and an image's noise does not depend on how the run is sharded."""
    out = torch.empty(stop - start, channels, image_size, image_size)
    for j, i in enumerate(range(start, stop)):
        g = torch.Generator().manual_seed(seed * 1_000_003 + i)
        out[j].normal_(generator=g)
    return out


class GraphedHeunSampler:
    """The doubled-batch Heun sampler for a fixed batch of `batch` images, captured as
    one CUDA graph (all ``2 * steps - 1`` model calls and the updates between them).

    ``sampler(labels, noise)`` copies the inputs into the graph's static buffers,
    replays it on the current stream and returns the static output buffer (valid
    until the next call; ``clone()`` it to keep it).  `autocast` is the dtype the
    model runs under (None: no autocast).  The model's weights are read in place at
    every replay, so parameter updates are seen; shapes, the step count and the
    guidance settings are fixed at capture.  Capture is preceded by one eager model
    call at the doubled batch (library handles and workspaces)."""

    def __init__(self, model, batch: int, *, image_size=256, noise_scale=1.0, steps=50, cfg_scale=1.0,
                 interval=(0.0, 1.0), num_classes=1000, t_eps=5e-2, prediction="clean",
                 autocast: torch.dtype | None = torch.bfloat16, device=None):
        device = torch.device(device if device is not None else torch.cuda.current_device())
        self.model, self.batch, self.noise_scale = model, batch, noise_scale
        self.kw = dict(num_classes=num_classes, cfg_scale=cfg_scale, interval=interval, t_eps=t_eps,
                       prediction=prediction)
        self.ts = _time_grid(steps, device)
        self.autocast = autocast
        self.noise = torch.zeros(batch, 3, image_size, image_size, device=device)
        self.labels = torch.zeros(batch, dtype=torch.long, device=device)
        self.graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            self._run(warm_up=True)  # one model call outside the capture: library handles, workspaces
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize(device)
        with torch.cuda.graph(self.graph):
            self.out = self._run()

    @torch.no_grad()
    def _run(self, warm_up: bool = False) -> torch.Tensor:
        ctx = (torch.autocast("cuda", dtype=self.autocast) if self.autocast is not None
               else contextlib.nullcontext())
        with ctx:
            if warm_up:
                t = torch.full((self.batch, 1, 1, 1), float(self.ts[0]), device=self.noise.device)
                return cfg_velocity_doubled(self.model, self.noise, t, self.labels, **self.kw)
            return _heun_loop(self.model, self.noise * self.noise_scale, self.labels, self.ts, self.kw)

    def __call__(self, labels: torch.Tensor, noise: torch.Tensor) -> torch.Tensor:
        if labels.numel() != self.batch or tuple(noise.shape) != tuple(self.noise.shape):
            raise ValueError(f"captured for {self.batch} images of {tuple(self.noise.shape[1:])}, got "
                             f"{labels.numel()} labels and noise {tuple(noise.shape)}")
        self.labels.copy_(labels.reshape(-1), non_blocking=True)
        self.noise.copy_(noise, non_blocking=True)
        self.graph.replay()
        return self.out


__all__ = ["sample_heun", "cfg_velocity_doubled", "image_noise", "GraphedHeunSampler"]
