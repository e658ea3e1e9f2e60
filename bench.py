#!/usr/bin/env python
"""LTHC interface benchmark on B200 (one JSON line on rank 0).

Step = one fused materialisation X_L = X_0 + sum_{l<12} P_l(dZ_l) over one batch
of BASELINE configuration 2 (B=64 per GPU, bf16 activations, fp32 write weights,
NHWC [64, 64, 64, 768] residual, 12 workspace updates [64, 256, 768]).  The
metric is algorithmic HBM bytes per second (1,107,886,080 B per step and GPU),
summed over GPUs (weak scaling: every rank runs its own batch, no collective on
the data path).  Inputs are 1.1 GB per step, larger than the 126 MB L2, so no L2
flush is needed between steps.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

``--impl reference`` times the CPU restatement of the reference's algorithm
(``oracle/``, all host threads) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import contextlib
import ctypes
import json
import os
import shutil
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

from flowmatching_lthc_b200 import dist as D  # noqa: E402
from flowmatching_lthc_b200 import workloads as W  # noqa: E402

METRIC = "LTHC read/write/materialise HBM GB/s vs peak"
UNIT = "GB/s"
FALLBACK_HBM_GBS = 6650.0
B_DEFAULT, G, C, L = 64, 16, 768, 12
TRAFFIC_FILE = ROOT / "profiles" / "materialise_fwd_b64_bf16.md"
SPIN_CYCLES = 2_000_000  # ~1 ms at the B200's clock: outside the timed region


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=4000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--batch", type=int, default=B_DEFAULT, help="images per GPU (BASELINE config 2: 64)")
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample duration")
    p.add_argument("--no-extras", action="store_true", help="skip the per-kernel and comparator measurements")
    p.add_argument("--op", default="materialise_fwd", choices=sorted(OPS),
                   help="the LTHC op timed as the step (default: the BASELINE config 2 materialisation)")
    p.add_argument("--no-model", action="store_true",
                   help="skip the LTHC-B/4 images/sec legs (forward, training step, sampling)")
    p.add_argument("--reference-gpu", action="store_true",
                   help="also time the reference's own model on the GPU (needs the reference package)")
    p.add_argument("--placement-sweep", action="store_true",
                   help="instead of the benchmark: the materialisation's GB/s over output / x0 placements "
                        "(swept forward and in reverse) and the per-launch times after an idle GPU")
    return p.parse_args()


def hbm_peak() -> tuple[float, str]:
    f = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(f.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic_per_launch() -> float | None:
    """dram bytes (read + write) per materialise launch at the bench config, from the
    committed ncu summary (line 'dram_bytes_per_launch: N')."""
    try:
        for line in TRAFFIC_FILE.read_text().splitlines():
            if line.strip().startswith("dram_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip().split()[0])
    except Exception:
        pass
    return None


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, interval_ms: int = 100):
        self.samples: list[tuple[float, list[str]]] = []
        self.proc = None
        exe = shutil.which("nvidia-smi")
        if not exe:
            return
        self.proc = subprocess.Popen([exe, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                      f"-lms={interval_ms}"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                     text=True)
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), [s.strip() for s in line.split(",")]))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(5)
            except Exception:
                self.proc.kill()
            self.thread.join(2)

    def summary(self, t0: float, t1: float, gpus: int) -> dict:
        rows = [s for t, s in self.samples if t0 <= t <= t1 and len(s) >= 9]
        note = None
        if not rows:
            rows = [s for _, s in self.samples if len(s) >= 9]
            note = "no sample fell inside the timed region; all samples of the run"
        rows = [s for s in rows if s[0].isdigit() and int(s[0]) < gpus]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "note": "nvidia-smi unavailable"}
        sm = [float(s[1]) for s in rows if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in rows if s[2].replace(".", "").isdigit()]
        reasons = sorted({name for s in rows for name, v in zip(self.REASONS, s[5:9]) if v.lower() == "active"})
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
               "reasons": reasons, "samples": len(rows)}
        if note:
            out["note"] = note
        return out


# ------------------------------------------------------------------ helpers
def time_device(fn, iters: int, stream: torch.cuda.Stream) -> float:
    """Average device time in ms of fn() over `iters` calls (CUDA events on `stream`)."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(iters):
        fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / iters


def host_link(h_src: torch.Tensor, d_buf: torch.Tensor, r: D.Rank, dev, stream) -> dict:
    """Pinned host<->device copy bandwidth of this rank while every rank copies at
    once (barrier-aligned): the ceiling of an end-to-end leg whose inputs and
    results cross the host link.  GB/s per rank, slowest rank."""
    n = min(h_src.numel(), d_buf.numel())
    src, dst = h_src.reshape(-1)[:n], d_buf.reshape(-1)[:n]
    nbytes = n * h_src.element_size()
    out = {}
    for name, fn in (("h2d", lambda: dst.copy_(src, non_blocking=True)),
                     ("d2h", lambda: src.copy_(dst, non_blocking=True))):
        fn()
        torch.cuda.synchronize()
        D.barrier()
        ms = D.reduce_max(time_device(fn, 3, stream), dev)
        out[f"{name}_gbs"] = round(nbytes / (ms / 1e3) / 1e9, 2)
    out["bytes_per_copy"] = nbytes
    out["aggregate_h2d_gbs"] = round(out["h2d_gbs"] * r.world, 1)
    out["aggregate_d2h_gbs"] = round(out["d2h_gbs"] * r.world, 1)
    return out


def host_threads() -> int:
    """All host threads this process may run on (torchrun sets OMP_NUM_THREADS=1,
    so the CPU legs set their thread count explicitly)."""
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_baseline_isolated(seconds: float) -> dict:
    """cpu_baseline() in a fresh child process.  Timed inside this process, after the
    CUDA legs, the same oracle ran at half its rate (CPU thread pools and driver
    threads of the GPU work still competing for the cores); a clean process
    measures it the way the reference arm does."""
    code = (f"import json, sys; sys.path.insert(0, {str(ROOT)!r}); import bench; "
            f"print(json.dumps(bench.cpu_baseline({float(seconds)!r})))")
    env = {k: v for k, v in os.environ.items() if k not in ("OMP_NUM_THREADS",)}
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=600)
    if res.returncode != 0:
        raise RuntimeError(f"CPU baseline child failed: {res.stderr[-400:]}")
    return json.loads(res.stdout.strip().splitlines()[-1])


def cpu_baseline(seconds: float) -> dict:
    """The oracle (CPU restatement of the reference's algorithm) on a bounded
    sample of the same workload, all host threads."""
    from oracle import lthc_oracle as O

    O.set_num_threads(host_threads())
    Bs = 4
    cfg = W.config2(B=Bs, seed=0)
    O.materialise(cfg["x0"], cfg["dz"], cfg["P"])
    n, t0 = 0, time.perf_counter()
    while True:
        O.materialise(cfg["x0"], cfg["dz"], cfg["P"])
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    by = W.materialise_bytes(Bs, G, C, L, 2) * n
    return {"value": round(by / el / 1e9, 4), "unit": UNIT, "cores": O.num_threads(), "kind": "port",
            "sample": f"{n} x materialise of B={Bs} (config 2 shapes, bf16) in {el:.1f} s on {O.num_threads()} threads",
            "scope": "one process on every host thread: the whole host CPU, compared with all GPUs of the job"}


def reference_eager_cpu(Bs: int, seconds: float) -> dict | None:
    """The reference's own CPU path for the materialisation, timed when the reference
    package is importable (LTHC_REFERENCE or baseline/_ref): its pure-torch loop of
    12 write_add calls (local_thc.py:1368-1372, 1275-1276) in torch eager on every
    host thread, bf16 as under autocast.  None when the package is absent."""
    for cand in (os.environ.get("LTHC_REFERENCE"), str(ROOT / "baseline" / "_ref")):
        if cand and (Path(cand) / "flowmatching_lthc").exists() and cand not in sys.path:
            sys.path.insert(0, cand)
    try:
        sys.dont_write_bytecode = True
        from flowmatching_lthc.models import local_thc as Lr
    except Exception:
        return None
    torch.set_num_threads(host_threads())
    cfg = W.config2(B=Bs, seed=0)
    writes = []
    for p in cfg["P"]:
        w = Lr.LayerLocalWrite(4 * G, G, C, C)
        with torch.no_grad():
            w.write_weight.copy_(p)
        writes.append(type("Blk", (), {"write": w})())
    holder = type("M", (), {"blocks": writes})()
    fn = Lr.SharedReadLocalTHCSharedAdaLNJiT.final_accumulate_reference
    with torch.no_grad():
        fn(holder, cfg["x0"], cfg["dz"])
        n, t0 = 0, time.perf_counter()
        while True:
            fn(holder, cfg["x0"], cfg["dz"])
            n += 1
            el = time.perf_counter() - t0
            if el >= seconds:
                break
    by = W.materialise_bytes(Bs, G, C, L, 2) * n
    return {"value": round(by / el / 1e9, 4), "unit": UNIT, "cores": torch.get_num_threads(), "kind": "reference",
            "sample": f"{n} x the reference's final_accumulate_reference (12 x write_add, torch eager) at B={Bs}, "
                      f"bf16, in {el:.1f} s"}


# ------------------------------------------------------------------ ops
def _op_inputs(B: int, dev, seed: int) -> dict:
    cfg = W.config2(B=B, device=dev, seed=seed)
    cfg["g"] = W.residual(B, G, C, seed=seed + 7, device=dev, dtype=torch.bfloat16)
    cfg["alpha"] = torch.softmax(torch.randn(C, 16, device=dev, generator=torch.Generator(device=dev).manual_seed(seed)),
                                 -1).to(torch.bfloat16)
    cfg["z"] = torch.randn(B, G * G, C, device=dev, dtype=torch.bfloat16)
    return cfg


def op_step(op: str, cfg: dict):
    """(step callable, algorithmic HBM bytes per step, kernel launches per step, kernel names)."""
    from flowmatching_lthc_b200 import ops

    B = cfg["B"]
    x0, dz, P, g, alpha, z = cfg["x0"], cfg["dz"], cfg["P"], cfg["g"], cfg["alpha"], cfg["z"]
    beta = P[0].to(torch.bfloat16)
    table = {
        "materialise_fwd": (lambda: ops.call(ops.materialise, x0, dz, P), W.materialise_bytes(B, G, C, L, 2), 1,
                            "broadcast_tma_kernel<bf16, 12, base>"),
        "materialise_bwd": (lambda: ops.call(ops.materialise_bwd, g, dz, P, True, True), W.materialise_bwd_bytes(B, G, C, L, 2), 2,
                            "matbwd_tc_kernel<bf16> + matbwd_tc_finalize_kernel"),
        "materialise_grad_dz": (lambda: ops.call(ops.materialise_grad_dz, g, P), W.materialise_grad_dz_bytes(B, G, C, L, 2),
                                1, "matbwd_tc_kernel<bf16> (grad_dz only)"),
        "materialise_grad_beta": (lambda: ops.call(ops.materialise_grad_beta, g, dz),
                                  W.materialise_grad_beta_bytes(B, G, C, L, 2), 2,
                                  "matbwd_tc_kernel<bf16> (grad_beta only) + matbwd_tc_finalize_kernel"),
        "read_fwd": (lambda: ops.call(ops.read, x0, alpha), W.read_bytes(B, G, C, 2, 2), 1, "pool_tma_kernel<bf16, 1, pool>"),
        "read_bwd": (lambda: ops.call(ops.read_bwd, x0, z, alpha, True, True), W.read_bwd_bytes(B, G, C, 2, 2), 2,
                     "broadcast_tma_kernel<bf16, 1, wgrad> (one pass) + reduce_partials_kernel"),
        "write_add_fwd": (lambda: ops.call(ops.write_add, x0, dz[0], beta), W.write_add_bytes(B, G, C, 2, 2), 1,
                          "broadcast_tma_kernel<bf16, 1, base>"),
        "lazy_fwd": (lambda: ops.call(ops.lazy_update, z, dz[0], alpha, beta), W.lazy_bytes(B * G * G, C, 2, 2), 1,
                     "lazy_fwd_kernel<bf16>"),
        "lazy_bwd": (lambda: ops.call(ops.lazy_update_bwd, z, dz[0], alpha, beta), W.lazy_bytes(B * G * G, C, 2, 2), 2,
                     "lazy_bwd_kernel<bf16> + lazy_bwd_finalize_kernel"),
    }
    if op == "embed_fwd":
        # patch embedding + shared read of BASELINE config 3's images (B, 3, 256, 256)
        gen = torch.Generator(device=x0.device).manual_seed(11)
        img = torch.randn(B, 3, 4 * 4 * G, 4 * 4 * G, device=x0.device, generator=gen)
        w1 = torch.randn(128, 3, 4, 4, device=x0.device, generator=gen) * 0.14
        w2 = torch.randn(C, 128, 1, 1, device=x0.device, generator=gen) * 0.09
        b2 = torch.randn(C, device=x0.device, generator=gen) * 0.1
        table["embed_fwd"] = (lambda: ops.call(ops.patch_embed_read, img, w1, w2, b2, alpha), W.embed_bytes(B, 4 * G, C), 1,
                              "patch_embed_read_kernel (tcgen05)")
    if op in ("branch_fwd", "branch_bwd"):
        # branch epilogue + lazy update on the workspace rows [B, 256, 768]; gate is a chunk of t6
        gen = torch.Generator(device=x0.device).manual_seed(13)
        attn = torch.randn(B, G * G, C, device=x0.device, generator=gen).to(torch.bfloat16)
        mlp = torch.randn(B, G * G, C, device=x0.device, generator=gen).to(torch.bfloat16)
        gate = (0.5 * torch.randn(B, 6 * C, device=x0.device, generator=gen)).to(torch.bfloat16).chunk(6, dim=-1)[5]
        gdz = torch.randn(B, G * G, C, device=x0.device, generator=gen).to(torch.bfloat16)
        n = B * G * G
        table["branch_fwd"] = (lambda: ops.call(ops.branch_lazy_update, z, attn, mlp, gate, alpha, beta),
                               W.branch_fwd_bytes(n, B, C, 2, 2), 1, "branch_lazy_fwd_kernel<bf16>")
        table["branch_bwd"] = (lambda: ops.call(ops.branch_lazy_update_bwd, gdz, z, attn, mlp, gate, alpha, beta),
                               W.branch_bwd_bytes(n, B, C, 2, 2), 2,
                               "branch_lazy_bwd_kernel<bf16> + branch_lazy_bwd_finalize_kernel")
    if op in ("final_fwd", "final_bwd"):
        # final-layer prologue on the materialised residual [B, 4096, 768] (FinalLayerSharedAdaLN)
        T = 16 * G * G
        xt, gm = x0.reshape(B, T, C), g.reshape(B, T, C)
        nw = torch.ones(C, device=x0.device) + 0.1 * torch.randn(C, device=x0.device)
        t2 = (0.5 * torch.randn(B, 2 * C, device=x0.device)).to(torch.bfloat16)
        sh, sc = t2.chunk(2, dim=1)
        table["final_fwd"] = (lambda: ops.call(ops.final_norm_modulate, xt, nw, sh, sc, 1e-6), W.final_fwd_bytes(B, T, C, 2), 1,
                              "final_norm_modulate_kernel<bf16, fwd>")
        table["final_bwd"] = (lambda: ops.call(ops.final_norm_modulate_bwd, gm, xt, nw, sc, 1e-6), W.final_bwd_bytes(B, T, C, 2),
                              2, "final_norm_modulate_kernel<bf16, bwd> + final_bwd_finalize_kernel")
    return table[op]


OPS = ("materialise_fwd", "materialise_bwd", "materialise_grad_dz", "materialise_grad_beta", "read_fwd", "read_bwd", "write_add_fwd", "lazy_fwd", "lazy_bwd",
       "final_fwd", "final_bwd", "embed_fwd", "branch_fwd", "branch_bwd")


# ------------------------------------------------------------------ model-level workloads
SAMPLE_IMAGES = 1024       # Heun-50, CFG 1.5, 1024 images sharded over the GPUs
SAMPLE_CHUNK = 512         # images per captured sampling graph (a doubled batch of 1024 per model call)


def _model(dev, seed: int = 1):
    """LTHC-B/4 (flowmatching_lthc_b200.model) with seeded random weights (every layer
    non-zero, so no work is trivially zero)."""
    from flowmatching_lthc_b200.model import build_model, fill_seeded_

    return fill_seeded_(build_model("lthc_b4_velocity"), seed).to(dev)


def _timed(step, steps: int, stream) -> float:
    """Device ms of `steps` calls of step(), max over ranks, barrier + sync on both sides."""
    D.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    e1.synchronize()
    D.barrier()
    return D.reduce_max(e0.elapsed_time(e1), stream.device)


def model_legs(r: D.Rank, dev, stream, reference_gpu: bool = False) -> dict:
    """Images/sec of the LTHC-B/4 model at N GPUs (whole-job aggregates, device time,
    max over ranks), bf16 autocast, seeded synthetic inputs:
      forward   BASELINE config 3: B = 64 per GPU;
      train     config 4: fwd + bwd + fused AdamW, 32 images per GPU; for N > 1 the
                gradients accumulate into one flat buffer averaged by a single NCCL
                all-reduce per step (dist.FlatGradients), with the step without any
                exchange, a bare all-reduce and PyTorch's DDP reported beside it;
      sample    config 5: Heun-50 CFG 1.5 (velocity target) of 1024 images, host-seeded
                per-image noise and labels sharded over the ranks, doubled batch,
                each chunk of <= 512 images one captured CUDA graph.
    With `reference_gpu` (needs the reference package importable), the reference's
    own model with identical weights is timed on the same inputs: forward and train
    step with its eager LTHC + Triton materialisation, sampling with its two-call
    sampler on chunks of <= 256 images (its Triton op's 32-bit offsets wrap above
    682 images per call)."""
    from flowmatching_lthc_b200.sampling import GraphedHeunSampler, image_noise

    out: dict = {}
    gen = torch.Generator(device=dev).manual_seed(2000 + r.rank)
    m = _model(dev)
    refm = _reference_model(dev) if reference_gpu else None

    # config 3: forward at B = 64 per GPU
    B = 64
    x = torch.randn(B, 3, 256, 256, device=dev, generator=gen)
    t = torch.rand(B, device=dev, generator=gen)
    y = torch.randint(0, 1000, (B,), device=dev, generator=gen)
    leg = {}
    for tag, net in (("ours", m), ("reference", refm)):
        if net is None:
            continue
        net.eval()

        def fwd(net=net):
            with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
                net(x, t, y)
        for _ in range(3):
            fwd()
        ms = _timed(fwd, 10, stream)
        leg[tag] = {"images_per_s": round(r.world * B * 10 / (ms / 1e3), 1), "ms_per_batch": round(ms / 10, 3)}
        if tag == "ours":
            # the same forward replayed from one CUDA graph (autocast weight cache off)
            def fwd_nc(net=net):
                with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16, cache_enabled=False):
                    net(x, t, y)
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                fwd_nc()
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                fwd_nc()
            for _ in range(3):
                graph.replay()
            gms = _timed(graph.replay, 10, stream)
            leg[tag] = {"images_per_s": round(r.world * B * 10 / (gms / 1e3), 1), "ms_per_batch": round(gms / 10, 3),
                        "path": "one CUDA graph per batch", "eager": leg[tag]}
            del graph
    out["forward"] = {"config": "BASELINE config 3: B=64 per GPU, bf16 autocast", "batch_per_gpu": B,
                      "steps": 10, **leg.pop("ours"), **({"reference_gpu": leg["reference"]} if leg else {})}

    # config 4: training step, 32 images per GPU
    B = 32
    x1 = torch.randn(B, 3, 256, 256, device=dev, generator=gen)
    e = torch.randn(B, 3, 256, 256, device=dev, generator=gen)
    t = torch.rand(B, device=dev, generator=gen)
    y = torch.randint(0, 1000, (B,), device=dev, generator=gen)
    tt = t.view(-1, 1, 1, 1)
    zt = tt * x1 + (1 - tt) * e
    v = (x1 - zt) / (1 - tt).clamp_min(0.05)
    leg = {}

    def make_step(net, opt, zero, exchange):
        def train():
            zero()
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = (v - net(zt, t, y)).float().square().mean()
            loss.backward()
            exchange()
            opt.step()
        return train

    def timed_train(step):
        for _ in range(3):
            step()
        ms = _timed(step, 10, stream)
        return {"images_per_s": round(r.world * B * 10 / (ms / 1e3), 1), "ms_per_step": round(ms / 10, 3)}

    # ours: gradients accumulate into one flat buffer, one all-reduce (mean) per step;
    # forward + backward and the update replayed from two CUDA graphs (the exchange
    # runs eagerly between them); the same step eagerly for comparison
    from flowmatching_lthc_b200.training import GraphedTrainStep, flow_matching_step
    m.train()
    opt = torch.optim.AdamW(m.parameters(), lr=1e-4, fused=True, capturable=True)
    fg = D.FlatGradients(m.parameters())
    eager = timed_train(make_step(m, opt, fg.zero_grad, fg.allreduce))
    graphed = GraphedTrainStep(flow_matching_step(m, fg.zero_grad, zt, t, y, v), opt.step)
    leg["ours"] = timed_train(lambda: graphed(fg.allreduce))
    leg["ours"]["path"] = "forward + backward and the AdamW update replayed from two CUDA graphs, exchange eager"
    leg["ours"]["eager"] = eager
    del graphed  # release the graphs' memory pool before the comparison steps
    if r.world > 1:
        # the same step without any exchange, one bare all-reduce of the gradient bytes,
        # and PyTorch's DistributedDataParallel (bucketed all-reduces during backward)
        leg["ours"]["ms_per_step_without_exchange"] = timed_train(make_step(m, opt, fg.zero_grad, lambda: None))[
            "ms_per_step"]
        fg.allreduce()
        leg["ours"]["allreduce_ms"] = round(_timed(fg.allreduce, 5, stream) / 5, 3)
        leg["ours"]["allreduce_bytes"] = fg.flat.numel() * 4
        ddp = torch.nn.parallel.DistributedDataParallel(m, device_ids=[r.local_rank], gradient_as_bucket_view=True)
        opt_d = torch.optim.AdamW(m.parameters(), lr=1e-4, fused=True)
        leg["ours"]["ddp"] = timed_train(make_step(ddp, opt_d, lambda: opt_d.zero_grad(set_to_none=True),
                                                   lambda: None))
        del ddp, opt_d
    del fg, opt
    if refm is not None:
        refm.train()
        net = (torch.nn.parallel.DistributedDataParallel(refm, device_ids=[r.local_rank]) if r.world > 1 else refm)
        opt = torch.optim.AdamW(refm.parameters(), lr=1e-4, fused=True)
        leg["reference"] = timed_train(make_step(net, opt, lambda: opt.zero_grad(set_to_none=True), lambda: None))
        del net, opt
    out["train_step"] = {"config": "BASELINE config 4: fwd+bwd+AdamW, 32 images per GPU, bf16 autocast" +
                         (f", data-parallel over {r.world} GPUs (one all-reduce of the flat gradient per step)"
                          if r.world > 1 else ""), "batch_per_gpu": B, "steps": 10,
                         **leg.pop("ours"), **({"reference_gpu": leg["reference"]} if leg else {})}
    # the training step changed the weights: sample with fresh ones
    m = _model(dev)
    if refm is not None:
        refm = _reference_model(dev)

    # config 5: Heun-50 CFG sampling of 1024 images sharded over the ranks
    lo, hi = D.shard(SAMPLE_IMAGES, r.rank, r.world)
    n = hi - lo
    labels_all = torch.randint(0, 1000, (SAMPLE_IMAGES,), generator=torch.Generator().manual_seed(5))
    chunks = [(a, min(a + SAMPLE_CHUNK, hi)) for a in range(lo, hi, SAMPLE_CHUNK)]
    noise = {c: image_noise(6, *c).pin_memory() for c in chunks}
    kw = dict(steps=50, cfg_scale=1.5, num_classes=1000, prediction="velocity")
    m.eval()
    samplers = {}
    for a, b in chunks:
        if b - a not in samplers:
            samplers[b - a] = GraphedHeunSampler(m, b - a, device=dev, **kw)
    outs = {c: torch.empty(c[1] - c[0], 3, 256, 256, pin_memory=True) for c in chunks}

    def sample():
        for c in chunks:
            img = samplers[c[1] - c[0]](labels_all[c[0]:c[1]].to(dev, non_blocking=True), noise[c].to(dev, non_blocking=True))
            outs[c].copy_(img, non_blocking=True)
    ms = _timed(sample, 1, stream)
    leg = {"images_per_s": round(SAMPLE_IMAGES / (ms / 1e3), 2), "ms": round(ms, 1)}
    if refm is not None:
        from flowmatching_lthc.sampling import sample_heun as ref_sample_heun

        refm.eval()

        def ref_sample():
            for a0 in range(lo, hi, 256):
                b0 = min(a0 + 256, hi)
                with torch.autocast("cuda", dtype=torch.bfloat16):
                    ref_sample_heun(refm, labels_all[a0:b0].to(dev), **kw)
        ms = _timed(ref_sample, 1, stream)
        leg["reference_gpu"] = {"images_per_s": round(SAMPLE_IMAGES / (ms / 1e3), 2), "ms": round(ms, 1),
                                "path": "reference two-call CFG sampler, eager LTHC + Triton materialisation, "
                                        "chunks of 256 images"}
    out["sample"] = {"config": "BASELINE config 5: Heun-50, CFG 1.5, 1024 images of 256x256, bf16 autocast",
                     "images": SAMPLE_IMAGES, "images_per_gpu": n, "chunk": SAMPLE_CHUNK,
                     "path": "doubled-batch CFG, whole loop of each chunk replayed as one CUDA graph, "
                             "host-seeded per-image noise (pinned) copied in, images copied out",
                     **leg}
    del samplers
    return out


def _reference_model(dev):
    """The reference's own released model class with the same seeded weights as _model
    (needs the reference package importable: LTHC_REFERENCE or baseline/_ref)."""
    for cand in (os.environ.get("LTHC_REFERENCE"), str(ROOT / "baseline" / "_ref")):
        if cand and (Path(cand) / "flowmatching_lthc").exists() and cand not in sys.path:
            sys.path.insert(0, cand)
    from flowmatching_lthc.models import build_model as ref_build

    from flowmatching_lthc_b200.model import fill_seeded_

    return fill_seeded_(ref_build("lthc_b4_velocity"), 1).to(dev)


# ------------------------------------------------------------------ placement sweep
def placement_sweep(dev) -> dict:
    """GB/s of the B = 64 materialisation with its output placed
    at 0..8 MB (256 KB steps) inside one buffer and x0 at 0..1 MB (64 KB steps),
    every other buffer fixed; each sweep runs in increasing and then decreasing
    order, so a drift over time (GPU warming up) and a dependence on placement can
    be told apart.  Then the per-launch GB/s of 400 back-to-back launches after the
    GPU idled for 1 s, 0.3 s and not at all."""
    from flowmatching_lthc_b200 import _lib

    cfg = W.config2(B=B_DEFAULT, device=dev, seed=1)
    dz, P = cfg["dz"], cfg["P"]
    nbytes = cfg["x0"].numel() * 2
    MB = 1 << 20
    big_out = torch.empty(nbytes + 9 * MB, dtype=torch.uint8, device=dev)
    big_x = torch.zeros(nbytes + 9 * MB, dtype=torch.uint8, device=dev)
    big_x[:nbytes].view(torch.bfloat16).copy_(cfg["x0"].reshape(-1))
    dzp, bp = _lib.ptr_array([t.data_ptr() for t in dz]), _lib.ptr_array([w.data_ptr() for w in P])
    stream = torch.cuda.current_stream(dev)
    nb = W.materialise_bytes(B_DEFAULT, G, C, L, 2)

    def run(xp, op):
        _lib.call("lthc_materialise_fwd", xp, dzp, bp, _lib.DTYPE_F32, L, op, B_DEFAULT, G, C, _lib.DTYPE_BF16,
                  stream.cuda_stream)

    def gbs(xp, op, it=30):
        for _ in range(5):
            run(xp, op)
        return round(nb / time_device(lambda: run(xp, op), it, stream) / 1e6, 1)

    out: dict = {}
    for name, offsets, fixed in (("out_offset_kb", range(0, 33), "x"), ("x0_offset_kb", range(0, 17), "out")):
        step = 256 * 1024 if fixed == "x" else 64 * 1024
        for order in ("increasing", "decreasing"):
            ks = list(offsets) if order == "increasing" else list(reversed(offsets))
            res = {}
            for k in ks:
                off = k * step
                res[off // 1024] = (gbs(big_x.data_ptr(), big_out.data_ptr() + off) if fixed == "x"
                                    else gbs(big_x.data_ptr() + off, big_out.data_ptr()))
            out[f"{name}_{order}"] = res
    for idle in (1.0, 0.3, 0.0):
        torch.cuda.synchronize()
        time.sleep(idle)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(401)]
        ev[0].record(stream)
        for i in range(400):
            run(big_x.data_ptr(), big_out.data_ptr())
            ev[i + 1].record(stream)
        ev[-1].synchronize()
        t = [ev[i].elapsed_time(ev[i + 1]) for i in range(400)]
        out[f"after_idle_{idle}s"] = {"first_5_launches_gbs": [round(nb / x / 1e6) for x in t[:5]],
                                      "launches_0_20_gbs": round(nb / (sum(t[:20]) / 20) / 1e6),
                                      "launches_20_400_gbs": round(nb / (sum(t[20:]) / 380) / 1e6)}
    return out


# ------------------------------------------------------------------ reference arm
def reference_arm(args, r: D.Rank) -> int:
    if not r.is_main:
        return 0
    from oracle import lthc_oracle as O

    O.set_num_threads(host_threads())
    per_step_s = 0.035  # measured B=4 cost of the oracle materialisation on 8 cores
    Bs = 4 if (args.steps + args.warmup) * per_step_s <= 120 else 1
    cfg = W.config2(B=Bs, seed=0)
    for _ in range(max(args.warmup, 1)):
        O.materialise(cfg["x0"], cfg["dz"], cfg["P"])
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.materialise(cfg["x0"], cfg["dz"], cfg["P"])
    el = time.perf_counter() - t0
    by = W.materialise_bytes(Bs, G, C, L, 2)
    value = by * args.steps / el / 1e9
    sample = (f"each step: oracle materialise of B={Bs} of config 2 (bf16 in/out, fp32 weights), "
              f"{O.num_threads()} host threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": r.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) residual, N(0,0.1) updates, N(0,0.02) weights)",
        "config": config_dict(args.batch, r.world),
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": O.num_threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    eager = reference_eager_cpu(Bs, 5.0)
    if eager is not None:
        line["reference_eager_cpu"] = eager
    print(json.dumps(line), flush=True)
    return 0


WORKLOADS = {
    "materialise_fwd": "materialise fwd X_L = X_0 + sum_l P_l(dZ_l), BASELINE config 2",
    "materialise_bwd": "materialise bwd (grad dZ_l and grad P_l from grad X_L), config 2 shapes",
    "materialise_grad_dz": "materialise bwd, pooling half alone (grad dZ_l from grad X_L), config 2 shapes",
    "materialise_grad_beta": "materialise bwd, weight-gradient half alone (grad P_l), config 2 shapes",
    "read_fwd": "shared read Z = R(X_0), config 2 shapes",
    "read_bwd": "read bwd (grad X_0 and grad alpha), config 2 shapes",
    "write_add_fwd": "write_add X + P(dZ), config 2 shapes",
    "lazy_fwd": "lazy update Z + Gamma*dZ, config 2 shapes",
    "lazy_bwd": "lazy update bwd, config 2 shapes",
    "final_fwd": "final-layer RMSNorm + AdaLN modulate on X_L [B, 4096, 768], config 2 shapes",
    "final_bwd": "final-layer RMSNorm + modulate bwd (grad X_L, grad norm weight / shift / scale), config 2 shapes",
    "branch_fwd": "branch output sum (dz_attn + gate*mlp_out) fused with the lazy update, config 2 workspace shapes",
    "branch_bwd": "its backward (grad dz_attn / mlp_out / gate / alpha / beta), config 2 workspace shapes",
    "embed_fwd": "patch embedding (4x4 conv 3->128, 1x1 conv 128->768) + shared read, config 3 images, tcgen05",
}


def config_dict(B: int, world: int, op: str = "materialise_fwd") -> dict:
    return {"workload": WORKLOADS[op], "op": op,
            "global_batch": B * world, "batch_per_gpu": B, "residual": [B, 4 * G, 4 * G, C],
            "updates": [L, B, G * G, C], "act_dtype": "bf16", "weight_dtype": "fp32",
            "parallelism": f"dp{world} (batch-sharded replicas, no data-path collective)",
            "l2": "inputs 1.1 GB per step per GPU > 126 MB L2; no flush needed"}


# ------------------------------------------------------------------ our arm
@contextlib.contextmanager
def _stdout_to_stderr():
    """Send everything written to file descriptor 1 (Python and C stdio alike) to
    stderr, so that stdout carries only the one JSON result line."""
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        yield
    finally:
        try:
            ctypes.CDLL(None).fflush(None)
        except OSError:
            pass
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)


def main() -> int:
    args = parse_args()
    r = D.from_env()

    if args.impl == "reference":
        return reference_arm(args, r)

    from flowmatching_lthc_b200 import ops

    if not torch.cuda.is_available():
        print(json.dumps({"impl": "ours", "error": "no CUDA device"}))
        return 1
    torch.cuda.set_device(r.local_rank)
    dev = torch.device("cuda", r.local_rank)
    with _stdout_to_stderr():  # the communicator set-up prints a version banner on stdout
        D.init("nccl", r, device=dev)
        D.barrier()
    stream = torch.cuda.current_stream(dev)
    B = args.batch
    if args.placement_sweep:
        if r.is_main:
            print(json.dumps({"placement_sweep": placement_sweep(dev), "kernel": "broadcast_tma_kernel<bf16, 12, base>",
                              "workload": WORKLOADS["materialise_fwd"]}), flush=True)
        D.barrier()
        D.shutdown()
        return 0

    cfg = _op_inputs(B, dev, seed=1000 + r.rank)
    step, bytes_step, launches, kernel = op_step(args.op, cfg)
    step()
    torch.cuda.synchronize()

    # The clock sampler starts first; the warm-up steps then run directly before
    # the timed region, so the GPU enters it busy rather than after an idle gap
    # (an idle GPU lowers its clocks, which a timed region of a few ms would see).
    sampler = ClockSampler() if r.is_main else None
    time.sleep(0.3 if sampler else 0)
    for _ in range(max(args.warmup, 3)):
        step()
    D.barrier()
    torch.cuda.synchronize()
    t_wall0 = time.time()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # A short device-side spin ahead of the start event: while it runs, the host
    # enqueues the first steps, so the timed region holds the K launches back to
    # back instead of starting with the host's dispatch of the first one (measured:
    # the first launch after a synchronise took 1.5-2.3x a steady one).
    torch.cuda._sleep(SPIN_CYCLES)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    ev1.synchronize()
    D.barrier()
    torch.cuda.synchronize()
    t_wall1 = time.time()
    ms_local = ev0.elapsed_time(ev1)
    ms = D.reduce_max(ms_local, dev)
    if sampler:
        sampler.stop()
    clocks = sampler.summary(t_wall0, t_wall1, r.world) if sampler else None

    value = r.world * bytes_step * args.steps / (ms / 1e3) / 1e9
    peak, peak_kind = hbm_peak()
    kernel_ms = ms_local / args.steps
    achieved = bytes_step / (kernel_ms / 1e3) / 1e9
    traffic = ncu_traffic_per_launch() if args.op == "materialise_fwd" else None
    if traffic is not None and B != B_DEFAULT:
        traffic *= B / B_DEFAULT

    # end to end through the public operator: pinned host inputs -> device -> host result
    e2e = None
    if args.op == "materialise_fwd":
        from flowmatching_lthc_b200.host import HostMaterialiser

        x0, dz, P = cfg["x0"], cfg["dz"], cfg["P"]
        h_x0 = x0.cpu().pin_memory()
        h_dz = [d.cpu().pin_memory() for d in dz]
        h_out = torch.empty_like(h_x0).pin_memory()
        hm = HostMaterialiser(dev, chunk=8, depth=3)
        e2e_step = lambda: hm(h_x0, h_dz, P, h_out)  # noqa: E731
        e2e_step()
        torch.cuda.synchronize()
        n_e2e = max(3, min(args.steps, 10))
        D.barrier()
        e2e_ms = D.reduce_max(time_device(e2e_step, n_e2e, stream), dev)
        h2d = h_x0.numel() * 2 + sum(d.numel() * 2 for d in h_dz)
        d2h = h_out.numel() * 2
        link = host_link(h_x0, x0, r, dev, stream)
        bound_ms = max(h2d / link["h2d_gbs"], d2h / link["d2h_gbs"]) / 1e6
        e2e = {"value": round(r.world * bytes_step / (e2e_ms / 1e3) / 1e9, 3), "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "ms_per_step": round(e2e_ms, 3), "steps": n_e2e,
               "path": ("pinned host buffers -> chunked cudaMemcpyAsync in / lthc_b200::materialise (C ABI) / "
                        "copy out on three streams (HostMaterialiser, 8-image chunks) -> host"),
               "host_link": {**link, "copy_bound_ms": round(bound_ms, 3),
                             "frac_of_copy_bound": round(bound_ms / e2e_ms, 3),
                             "note": (f"pinned copies measured with all {r.world} ranks copying at once; the bound "
                                      "assumes the two directions fully overlap")}}
        del h_x0, h_dz, h_out, hm

    extras = {}
    if r.world == 1 and not args.no_extras:
        extras = measure_kernels(cfg, stream, peak)

    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": r.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) residual, N(0,0.1) updates, N(0,0.02) fp32 weights; no dataset)",
        "config": config_dict(B, r.world, args.op),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": UNIT,
                     "frac": round(achieved / peak, 4), "traffic": traffic, "peak_source": f"{peak_kind} hbm_gbs",
                     "kernel": kernel, "algorithmic_bytes_per_launch": bytes_step},
        "cpu_baseline": None,
        "e2e": e2e,
        "gpu_launches": args.steps * launches,
        "clocks": clocks,
    }
    if extras:
        line["kernels"] = extras.get("kernels")
        line["comparators"] = extras.get("comparators")
    if args.op == "materialise_fwd" and not args.no_model:
        del cfg, step, extras
        torch.cuda.empty_cache()
        line["images_per_s"] = model_legs(r, dev, stream, reference_gpu=args.reference_gpu)
        line["gpu_launches_note"] = "gpu_launches counts the headline materialisation steps only"
    if r.is_main and r.world == 1 and args.op == "materialise_fwd":
        line["cpu_baseline"] = cpu_baseline_isolated(args.cpu_seconds)
    if r.is_main:
        print(json.dumps(line), flush=True)
    D.barrier()
    D.shutdown()
    return 0


def measure_kernels(cfg: dict, stream, peak) -> dict:
    """Device-timed GB/s of every LTHC op at B=64 bf16 (informational; not the
    headline), plus the reference's Triton ops on the same inputs when the
    reference package is installed under baseline/_ref."""
    out: dict = {"kernels": {}, "comparators": {}}
    iters = 20
    for op in OPS:
        fn, nbytes, launches, _ = op_step(op, cfg)
        fn()
        ms = time_device(fn, iters, stream)
        # host cost of one eager call (dispatch + ctypes), and device time of the
        # same calls replayed from a CUDA graph (no host gaps between launches)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(iters):
            fn()
        host_us = (time.perf_counter() - t0) / iters * 1e6
        torch.cuda.synchronize()
        graph_ms = None
        try:
            side = torch.cuda.Stream()
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                fn()
            stream.wait_stream(side)
            torch.cuda.synchronize()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                for _ in range(10):
                    fn()
            gr.replay()
            torch.cuda.synchronize()
            graph_ms = time_device(gr.replay, 5, stream) / 10
            del gr
        except Exception as e:  # capture is an extra measurement, not the headline
            graph_ms = f"capture failed: {type(e).__name__}"
        best = min(ms, graph_ms) if isinstance(graph_ms, float) else ms
        out["kernels"][op] = {"ms": round(ms, 4), "gbs": round(nbytes / (best / 1e3) / 1e9, 1),
                              "frac": round(nbytes / (best / 1e3) / 1e9 / peak, 4), "bytes": nbytes,
                              "launches": launches, "eager_ms": round(ms, 4),
                              "graph_ms": round(graph_ms, 4) if isinstance(graph_ms, float) else graph_ms,
                              "host_us_per_call": round(host_us, 1)}

    B, x0, dz, P, g = cfg["B"], cfg["x0"], cfg["dz"], cfg["P"], cfg["g"]
    # the reference's eager epilogue + lazy update (local_thc.py:321-323, 1326-1328):
    # four elementwise torch kernels plus the gamma reduction, on the same inputs
    gen = torch.Generator(device=x0.device).manual_seed(13)
    attn = torch.randn(B, G * G, C, device=x0.device, generator=gen).to(torch.bfloat16)
    mlp = torch.randn(B, G * G, C, device=x0.device, generator=gen).to(torch.bfloat16)
    gate = (0.5 * torch.randn(B, 6 * C, device=x0.device, generator=gen)).to(torch.bfloat16).chunk(6, dim=-1)[5]
    alpha, beta, z = cfg["alpha"], P[0].to(torch.bfloat16), cfg["z"]

    def eager_branch():
        d = attn + gate.unsqueeze(1) * mlp
        return d, z + (alpha * beta).sum(-1)[None, None, :] * d

    eager_branch()
    ms = time_device(eager_branch, iters, stream)
    nb = W.branch_fwd_bytes(B * G * G, B, C, 2, 2)
    out["comparators"]["eager_branch_epilogue_lazy"] = {
        "ms": round(ms, 4), "gbs": round(nb / (ms / 1e3) / 1e9, 1),
        "speedup_of_ours": round(ms / out["kernels"]["branch_fwd"]["ms"], 3)}
    ref = ROOT / "baseline" / "_ref"
    if (ref / "flowmatching_lthc").exists():
        try:
            sys.path.insert(0, str(ref))
            import flowmatching_lthc.models.local_thc  # noqa: F401  (registers jit_thc:: ops)

            f = torch.ops.jit_thc.final_accumulate_b4_12_traceable
            fn = lambda: f(x0, *dz, *P)  # noqa: E731
            fn()
            ms = time_device(fn, iters, stream)
            nb = W.materialise_bytes(B, G, C, L, 2)
            out["comparators"]["triton_final_accumulate_b4_12"] = {
                "ms": round(ms, 4), "gbs": round(nb / (ms / 1e3) / 1e9, 1),
                "speedup_of_ours": round(ms / out["kernels"]["materialise_fwd"]["ms"], 3)}
            gdz_op = torch.ops.jit_thc.final_accumulate_b4_12_grad_dz_ptr
            gb_op = torch.ops.jit_thc.final_accumulate_b4_12_grad_beta_ptr
            fnb = lambda: (gdz_op(g, *P), gb_op(g, *dz))  # noqa: E731
            fnb()
            ms = time_device(fnb, iters, stream)
            nb = W.materialise_bwd_bytes(B, G, C, L, 2)
            out["comparators"]["triton_final_accumulate_b4_12_bwd"] = {
                "ms": round(ms, 4), "gbs": round(nb / (ms / 1e3) / 1e9, 1),
                "speedup_of_ours": round(ms / out["kernels"]["materialise_bwd"]["ms"], 3)}
        except Exception as e:  # the reference's own Triton path
            out["comparators"]["error"] = f"{type(e).__name__}: {str(e)[:200]}"
    else:
        out["comparators"]["note"] = "reference package not installed under baseline/_ref"
    return out


if __name__ == "__main__":
    sys.exit(main())
