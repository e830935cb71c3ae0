#!/usr/bin/env python
"""Benchmark of the encode-and-render hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Workloads (seeded synthetic inputs; no dataset is involved):
  render  config 1: one 768x768 image, 92,160 splats (seed 1), render_alpha_octave(odds=True) forward +
          backward of an L2 loss against a seeded target.  One step = one image.
Multi-GPU: every rank runs its own images (no collective on the data path; weak scaling); the timed
region is bracketed by a barrier + synchronize and the max over ranks is reported.

--impl reference times the reference's algorithm on the host CPU (the C oracle restating the
reference's renderer, all host threads) on the same workload, printed with "impl": "reference".
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "768² encode+render images/s at 1/2/4/8 B200; render fwd+bwd ms/image"
L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return dict(hbm_gbs=d.get("hbm_gbs", 6650.0), bf16_tflops=d.get("bf16_tflops", 1590.0),
                    bf16_tflops_sustained=d.get("bf16_tflops_sustained", 1400.0), source="measured")
    return dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0, source="fallback")


# ------------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.f = None

    def __enter__(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "50"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.06)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.f is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.f.flush()
        rows = [r.split(",") for r in Path(self.f.name).read_text().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            r = [x.strip() for x in r]
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except ValueError:
                continue
            for n, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------------------------------ workloads
class RenderWorkload:
    """Config 1: render_alpha_octave(odds) forward + L2 backward of one 768^2 image, 92,160 splats."""

    name = "render"
    H = W = 768
    N = 92160

    def __init__(self, dev):
        import torch

        from gaussian_2d_splat_encoder_b200 import synth
        from gaussian_2d_splat_encoder_b200 import render_triton as rt

        self.torch, self.rt, self.dev = torch, rt, dev
        s = synth.synth_splats_cfg1(self.N, self.H, self.W, seed=1)
        self.host = {k: v.contiguous().pin_memory() for k, v in s.items()}
        self.keys = ("mu", "log_scale", "color", "opacity", "bg", "theta")
        self.dev_in = {k: v.to(dev) for k, v in s.items()}
        self.leaves = [self.dev_in[k].clone().requires_grad_(True) for k in self.keys]

    def step(self, leaves=None, target=None):
        torch, rt = self.torch, self.rt
        L = self.leaves if leaves is None else leaves
        tgt = self.dev_in["target"] if target is None else target
        out = rt.render_alpha_octave(L[0], L[1], L[2], L[3], L[4], self.H, self.W, theta=L[5], odds=True)
        loss = (out - tgt).square().mean()
        grads = torch.autograd.grad(loss, L)
        return loss, grads

    def e2e_step(self, out_bufs):
        """Host (pinned) -> device copy of the step's inputs, the step, device -> host of loss + grads."""
        torch = self.torch
        L = [self.host[k].to(self.dev, non_blocking=True).requires_grad_(True) for k in self.keys]
        tgt = self.host["target"].to(self.dev, non_blocking=True)
        loss, grads = self.step(L, tgt)
        for o, g in zip(out_bufs, grads):
            o.copy_(g, non_blocking=True)
        out_bufs[-1].copy_(loss.detach().reshape(1), non_blocking=True)

    def e2e_buffers(self):
        torch = self.torch
        bufs = [torch.empty(self.host[k].shape, dtype=torch.float32).pin_memory() for k in self.keys]
        bufs.append(torch.empty(1).pin_memory())
        return bufs

    def io_bytes(self):
        h2d = sum(self.host[k].numel() * 4 for k in self.keys) + self.host["target"].numel() * 4
        d2h = sum(self.host[k].numel() * 4 for k in self.keys) + 4
        return h2d, d2h

    def pixel_pairs(self, lib):
        """Algorithmic units of the compositing kernels: (tile, splat) pairs x 64 pixels, summed over
        the octaves, read back from one forward's binning."""
        import ctypes as C

        from gaussian_2d_splat_encoder_b200 import _lib
        from gaussian_2d_splat_encoder_b200.render_triton import _desc

        torch = self.torch
        d = _desc(mode=_lib.MODE_OCTAVE, B=1, N=self.N, C=3, H=self.H, W=self.W, TILE=8, odds=True, has_theta=True,
                  cutoff=3.0, base_texels=8.0, max_octaves=6, max_pairs=48_000_000)
        d.pair_capacity = lib.gs_render_pair_bound(C.byref(d))
        nb = lib.gs_render_workspace_size(C.byref(d), 0)
        ws = torch.empty(nb, dtype=torch.uint8, device=self.dev)
        out = torch.empty(1, 3, self.H, self.W, device=self.dev)
        f = [self.dev_in[k].contiguous() for k in self.keys]
        _lib.check(lib.gs_render_fwd(C.byref(d), *[_lib.ptr(t) for t in f], _lib.ptr(out), _lib.ptr(ws), nb,
                                     _lib.stream_of(self.dev)))
        torch.cuda.synchronize()
        tot = C.c_int64(0)
        _lib.check(lib.gs_render_debug_bins(C.byref(d), _lib.ptr(ws), C.byref(tot), None, None, None, None, None))
        return int(tot.value), int(tot.value) * 64

    @classmethod
    def config(cls):
        return {"workload": "config 1: render_alpha_octave(odds=True) fwd + L2 bwd, 768x768, 92,160 splats "
                            "(seed 1)", "images_per_step_per_gpu": 1, "H": cls.H, "W": cls.W, "splats": cls.N,
                "l2": "flushed between timed steps (256 MB write, outside the timed events)"}

    @classmethod
    def cpu_inputs(cls):
        from gaussian_2d_splat_encoder_b200 import synth

        return {k: v.numpy() for k, v in synth.synth_splats_cfg1(cls.N, cls.H, cls.W, seed=1).items()}

    @classmethod
    def cpu_step(cls, O, s):
        """One step of the reference's algorithm on the host: forward, then backward of the L2 loss."""
        out = O.render_alpha_octave(s["mu"], s["log_scale"], s["color"], s["opacity"], s["bg"], cls.H, cls.W,
                                    theta=s["theta"], odds=True)
        g = (2.0 / out.size) * (out - s["target"])
        O.render_alpha_octave(s["mu"], s["log_scale"], s["color"], s["opacity"], s["bg"], cls.H, cls.W,
                              theta=s["theta"], odds=True, grad_out=g)


WORKLOADS = {"render": RenderWorkload}


# ------------------------------------------------------------------------------------------ CPU side
def cpu_baseline(workload_cls, steps: int, budget_s: float = 20.0):
    """The reference's algorithm on the host cores (C oracle, all threads): images/s over a bounded
    sample of whole steps."""
    from oracle import oracle as O

    O.build()
    s = workload_cls.cpu_inputs()
    times = []
    t_all = time.perf_counter()
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        workload_cls.cpu_step(O, s)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > budget_s:
            break
    per = statistics.mean(times)
    return {"value": 1.0 / per, "unit": "images/s", "cores": O.num_threads(), "kind": "port",
            "sample": f"{len(times)} whole {workload_cls.name} steps (768x768, fwd+bwd) on the C oracle, "
                      f"{O.num_threads()} OpenMP threads, os.cpu_count()={os.cpu_count()}"}


# ------------------------------------------------------------------------------------------ main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="render")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    W = max(3, args.warmup)
    K = max(1, args.steps)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    wcls = WORKLOADS[args.workload]

    if args.impl == "reference":
        if rank != 0:
            return
        r = cpu_baseline(wcls, K, budget_s=150.0)
        line = {"metric": METRIC, "value": r["value"], "unit": "images/s", "n_gpus": args.gpus, "steps": K,
                "warmup": W, "ms_per_step": 1000.0 / r["value"], "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "fp32", "data": "synthetic", "impl": "reference",
                "config": wcls.config(),
                "cpu_baseline": r,
                "e2e": {"value": r["value"], "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist

    from gaussian_2d_splat_encoder_b200 import _lib

    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lib = _lib.load()
    wl = wcls(dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    for _ in range(W):
        wl.step()
    barrier()

    # device-resident timed region: per-step events, L2 flushed between steps outside the events
    lib.gs_profile_enable(1)
    l0 = lib.gs_kernel_launches()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    idx = int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local]) \
        if os.environ.get("CUDA_VISIBLE_DEVICES") else local
    with ClockSampler(idx) as clk:
        for i in range(K):
            flush.zero_()
            ev[i][0].record()
            wl.step()
            ev[i][1].record()
        torch.cuda.synchronize()
    launches = lib.gs_kernel_launches() - l0
    lib.gs_profile_enable(0)
    import ctypes as C

    ms_st = (C.c_double * 8)()
    cnt_st = (C.c_int64 * 8)()
    _lib.check(lib.gs_profile_collect(ms_st, cnt_st))
    step_ms = [a.elapsed_time(b) for a, b in ev]
    tot_ms = sum(step_ms)
    if world > 1:
        t = torch.tensor([tot_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        tot_ms = float(t.item())
    barrier()

    # end-to-end through the public API with host buffers
    bufs = wl.e2e_buffers()
    for _ in range(2):
        wl.e2e_step(bufs)
    barrier()
    Ke = max(3, min(K, 50))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(Ke):
        wl.e2e_step(bufs)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    pairs, pp = wl.pixel_pairs(lib)
    images = K * world
    value = images / (tot_ms / 1000.0)
    e2e_val = Ke * world / (e2e_ms / 1000.0)
    h2d, d2h = wl.io_bytes()
    clocks = clk.summary()
    f_mhz = clocks["sm_mhz"] or 1965.0
    # roofline of the dominant kernel (fields backward): FP32-bound, 40 FP32 lane-ops + 2 SFU per
    # pixel-pair (algorithmic count); peak = 148 SMs x 128 FP32 lanes x the sampled SM clock.
    ms_fwd = ms_st[1] / max(cnt_st[1], 1)
    ms_bwd = ms_st[4] / max(cnt_st[4], 1)
    fp32_peak = 148 * 128 * f_mhz * 1e6 / 1e9  # Gop/s
    sfu_peak = 148 * 16 * f_mhz * 1e6 / 1e9
    bwd_ach = 40.0 * pp / (ms_bwd * 1e-3) / 1e9
    fwd_ach_sfu = 3.0 * pp / (ms_fwd * 1e-3) / 1e9
    stages = {n: {"ms_per_call": ms_st[i] / max(cnt_st[i], 1), "calls": int(cnt_st[i])}
              for i, n in enumerate(("binning", "fields_fwd", "composite", "composite_bwd+adjoint", "fields_bwd",
                                     "finalize"))}
    pk = peaks()
    line = {
        "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": tot_ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32", "data": "synthetic", "config": {**wl.config(), "parallelism": f"dp{world} (image per GPU, "
                                                                                      "no collective)"},
        "render_fwd_bwd_ms_per_image": tot_ms / K,
        "roofline": {"bound": "fp32", "kernel": "k_fields_bwd", "achieved": bwd_ach, "peak": fp32_peak,
                     "unit": "Gop/s (FP32 lane-ops)", "frac": bwd_ach / fp32_peak, "traffic": None,
                     "units_per_launch": pp, "ops_per_unit": 40,
                     "peak_source": f"148 SMs x 128 FP32 lanes x {f_mhz:.0f} MHz (median SM clock sampled during "
                                    "the timed region); MEASURED_PEAKS.json has no FP32/SFU figure"},
        "roofline_fields_fwd": {"bound": "sfu", "achieved": fwd_ach_sfu, "peak": sfu_peak, "unit": "Gop/s (MUFU)",
                                "frac": fwd_ach_sfu / sfu_peak, "ops_per_unit": 3, "units_per_launch": pp},
        "stages_ms": stages, "pairs": pairs, "pixel_pairs": pp,
        "clocks": clocks, "gpu_launches": int(launches),
        "e2e": {"value": e2e_val, "unit": "images/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "peaks": pk,
    }
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(wcls, 3)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
