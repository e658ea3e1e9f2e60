"""Materialisation from host (pinned) buffers with the transfers pipelined.

A caller whose X_0 and workspace updates live in host memory (and who wants X_L
back in host memory) pays two PCIe transfers around a short kernel.  Done in
sequence, the host->device copy, the kernel and the device->host copy add up.
``materialise_from_host`` splits the batch into chunks and runs three streams:
copies in, the fused materialisation, copies out, so that the two PCIe
directions and the kernel overlap; the total approaches the larger of the two
transfer times.  Device staging buffers (a small ring of chunk-sized sets) are
allocated once per shape through the PyTorch caching allocator and reused.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops


@dataclass
class _Ring:
    x0: list
    dz: list


class HostMaterialiser:
    """Pipelined X_L = X_0 + sum_l P_l(dZ_l) for pinned host tensors.

    ``x0_host`` [B, 4G, 4G, C] and every ``dz_host[l]`` [B, G*G, C] must be pinned
    CPU tensors of one dtype; ``betas`` are device tensors [C, 16]; the result is
    written into the pinned ``out_host``.  ``chunk`` images are moved per stage and
    ``depth`` chunk-sized device buffer sets are kept in flight."""

    def __init__(self, device: torch.device | int | None = None, chunk: int = 8, depth: int = 3):
        if device is None:
            device = torch.cuda.current_device()
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        self.chunk = chunk
        self.depth = depth
        self.s_in = torch.cuda.Stream(self.device)
        self.s_comp = torch.cuda.Stream(self.device)
        self.s_out = torch.cuda.Stream(self.device)
        self._ring: _Ring | None = None
        self._key = None

    def _buffers(self, x0_host: torch.Tensor, dz_host: list[torch.Tensor]) -> _Ring:
        key = (tuple(x0_host.shape[1:]), tuple(dz_host[0].shape[1:]), len(dz_host), x0_host.dtype)
        if self._ring is None or self._key != key:
            cx = (self.chunk,) + tuple(x0_host.shape[1:])
            cz = (self.chunk,) + tuple(dz_host[0].shape[1:])
            kw = dict(device=self.device, dtype=x0_host.dtype)
            self._ring = _Ring(x0=[torch.empty(cx, **kw) for _ in range(self.depth)],
                               dz=[[torch.empty(cz, **kw) for _ in dz_host] for _ in range(self.depth)])
            self._key = key
        return self._ring

    def __call__(self, x0_host: torch.Tensor, dz_host: list[torch.Tensor], betas: list[torch.Tensor],
                 out_host: torch.Tensor) -> torch.Tensor:
        if not (x0_host.is_pinned() and out_host.is_pinned() and all(t.is_pinned() for t in dz_host)):
            raise ValueError("materialise_from_host needs pinned host tensors (tensor.pin_memory())")
        B = x0_host.shape[0]
        ring = self._buffers(x0_host, dz_host)
        caller = torch.cuda.current_stream(self.device)
        for s in (self.s_in, self.s_comp, self.s_out):
            s.wait_stream(caller)
        free = [None] * self.depth  # event: the set's previous chunk has been copied out
        done = []
        for i, b0 in enumerate(range(0, B, self.chunk)):
            n = min(self.chunk, B - b0)
            k = i % self.depth
            x0_d = ring.x0[k][:n]
            dz_d = [t[:n] for t in ring.dz[k]]
            with torch.cuda.stream(self.s_in):
                if free[k] is not None:
                    self.s_in.wait_event(free[k])
                x0_d.copy_(x0_host[b0:b0 + n], non_blocking=True)
                for dst, src in zip(dz_d, dz_host):
                    dst.copy_(src[b0:b0 + n], non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record(self.s_in)
            with torch.cuda.stream(self.s_comp):
                self.s_comp.wait_event(ev_in)
                out_d = ops.call(ops.materialise, x0_d, dz_d, betas)
                ev_c = torch.cuda.Event()
                ev_c.record(self.s_comp)
            with torch.cuda.stream(self.s_out):
                self.s_out.wait_event(ev_c)
                out_host[b0:b0 + n].copy_(out_d, non_blocking=True)
                ev_o = torch.cuda.Event()
                ev_o.record(self.s_out)
                out_d.record_stream(self.s_out)
            free[k] = ev_o
            done.append(ev_o)
        if done:
            caller.wait_event(done[-1])  # copies out run in order on one stream
        return out_host


def materialise_from_host(x0_host, dz_host, betas, out_host, chunk: int = 8, depth: int = 3):
    """One-shot convenience wrapper around HostMaterialiser."""
    return HostMaterialiser(chunk=chunk, depth=depth)(x0_host, dz_host, betas, out_host)


__all__ = ["HostMaterialiser", "materialise_from_host"]
