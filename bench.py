#!/usr/bin/env python
"""Benchmark of the encode-and-render hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Workloads (seeded synthetic inputs; no dataset is involved):
  encode_render (default) configs 2/3: 768x768 test cards (seeds 100-163, 500 shapes, 150 strokes), the
          released checkpoint when a local copy exists (weights/encoder_golden_d256.pt) else random init
          (seed 0); one step = one image per GPU: EfficientGaussianEncoder forward (bf16 tensor cores, with
          its internal 384^2 coarse render) + render_alpha_octave(odds=True) at 768^2 (fp32).
  render  config 1: one 768x768 image, 92,160 splats (seed 1): render_alpha_octave(odds=True) forward +
          backward of an L2 loss against a seeded target.  Its ms/image is also reported by every
          encode_render line ("render_fwd_bwd_ms_per_image").
Multi-GPU: every rank runs its own images (no collective on the data path; weak scaling); the timed
region is bracketed by a barrier + synchronize and the max over ranks is reported.

--impl reference times the reference's algorithm on the host CPU (fp32 torch-CPU restatement of the
encoder + the C oracle of the renderer, all host threads) on the same workload; rank 0 alone prints it.
"""

from __future__ import annotations

import argparse
import ctypes as C
import datetime
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
FIT_METRIC = "config 4: 2048^2 fitting step (render fwd+bwd + NCCL reduce-scatter + sharded Adam + all-gather) steps/s"
L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2
# dram__bytes_read.sum + dram__bytes_write.sum of the forward field kernels of one encode+render step
# (ncu, profiles/fields_fwd_encode_render_768.md): 3.81 MB (coarse render, k_fields_deep8) + 7.93 MB (final
# render, k_fields_w8) read, nothing written back inside the launches (the field planes stay in L2)
FIELDS_FWD_TRAFFIC = 11.74e6
STAGE_NAMES = {0: "binning", 1: "fields_fwd", 2: "composite", 3: "composite_bwd+adjoint", 4: "fields_bwd",
               5: "finalize", 6: "enc_binning", 7: "enc_fields_fwd", 8: "enc_prep", 9: "conv1", 10: "conv2", 11: "conv3", 12: "conv4_decoder",
               13: "heads", 14: "enc_gn_concat_cond", 15: "enc_coarse_render"}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return dict(hbm_gbs=d.get("hbm_gbs", 6650.0), bf16_tflops=d.get("bf16_tflops", 1590.0),
                    bf16_tflops_sustained=d.get("bf16_tflops_sustained", 1400.0), source="measured")
    return dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0, source="fallback")


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled during the timed region.

    Primary source: NVML (the library nvidia-smi reads) polled every 2 ms from a host thread, so even a
    timed region of a few tens of milliseconds carries many samples; only samples taken inside
    `window()` count.  Fallback when NVML cannot be opened: an `nvidia-smi --query-gpu ... -lms 50` process
    started (and waited on until its first row) before the region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits that the run reports (hardware power brake is a form of hw_slowdown)
    REASON_BITS = (("hw_slowdown", 0x8), ("hw_slowdown", 0x80), ("hw_thermal_slowdown", 0x40),
                   ("sw_thermal_slowdown", 0x20), ("sw_power_cap", 0x4))
    PERIOD_S = 0.002

    def __init__(self, gpu_index: int, uuid: str | None = None, nvml=None):
        self.idx, self.uuid, self.nvml = gpu_index, uuid, nvml
        self.proc, self.f, self.thread, self.handle = None, None, None, None
        self.samples, self.win, self.max_mhz = [], None, None
        self._stop = None

    # ---- NVML path
    def _open_nvml(self):
        import threading

        nv = self.nvml
        if nv is None:
            import pynvml as nv
        nv.nvmlInit()
        h = None
        if self.uuid:  # the CUDA device's own UUID: immune to CUDA_VISIBLE_DEVICES / ordering differences
            try:
                h = nv.nvmlDeviceGetHandleByUUID("GPU-" + self.uuid)
            except Exception:
                h = None
        if h is None:
            h = nv.nvmlDeviceGetHandleByIndex(self.idx)
        self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        self.nvml, self.handle = nv, h
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                try:
                    t = time.perf_counter()
                    mhz = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((t, float(mhz), int(rs)))
                except Exception:
                    break
                self._stop.wait(self.PERIOD_S)

        self.thread = threading.Thread(target=run, name="clock-sampler", daemon=True)
        self.thread.start()

    # ---- nvidia-smi fallback
    def _open_smi(self):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                      "-i", str(self.idx), "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
        t0 = time.time()
        while time.time() - t0 < 5.0 and self.proc.poll() is None:  # first row written before timing starts
            if Path(self.f.name).stat().st_size > 0:
                break
            time.sleep(0.02)

    def __enter__(self):
        try:
            self._open_nvml()
        except Exception:
            self.thread = None
            try:
                self._open_smi()
            except Exception:
                self.proc = None
        return self

    def window(self):
        sampler = self

        class _Win:
            def __enter__(self):
                sampler.win = [time.perf_counter(), None]

            def __exit__(self, *a):
                sampler.win[1] = time.perf_counter()

        return _Win()

    def __exit__(self, *a):
        if self.thread is not None:
            self._stop.set()
            self.thread.join(timeout=5)
            try:
                self.nvml.nvmlShutdown()
            except Exception:
                pass
        if self.proc is not None:
            time.sleep(0.06)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.thread is not None:
            rows = list(self.samples)
            if self.win and self.win[1] is not None:
                inside = [r for r in rows if self.win[0] <= r[0] <= self.win[1]]
                rows = inside or [r for r in rows if r[0] >= self.win[0]][:1]
            reasons = {n for _, _, rs in rows for n, bit in self.REASON_BITS if rs & bit}
            sm = [mhz for _, mhz, _ in rows]
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                    "reasons": sorted(reasons), "samples": len(sm), "source": "nvml, 2 ms, inside the timed region"}
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
                "samples": len(sm), "source": "nvidia-smi -lms 50"}


# ------------------------------------------------------------------------------------------ workloads
def _load_encoder(dev=None):
    """The released checkpoint when a local copy exists, else the reference architecture with random
    init (torch.manual_seed(0)); returns (module, description)."""
    import torch

    from gaussian_2d_splat_encoder_b200.efficient_encoder import EfficientGaussianEncoder

    sys.path.insert(0, str(ROOT / "tests"))
    from enc_util import GOLDEN_CFG, load_golden

    m = load_golden(EfficientGaussianEncoder)
    desc = "released checkpoint encoder_golden_d256.pt"
    if m is None:
        torch.manual_seed(0)
        m = EfficientGaussianEncoder(**GOLDEN_CFG).eval()
        desc = "reference architecture, random init (torch.manual_seed(0))"
    if dev is not None:
        m = m.to(dev)
    return m, desc


class EncodeRenderWorkload:
    name = "encode_render"
    metric, unit, scaling = METRIC, "images/s", "weak"
    H = W = 768
    SEEDS = list(range(100, 164))

    def __init__(self, dev, rank=0, world=1):
        import torch

        from gaussian_2d_splat_encoder_b200 import pipeline, synth

        self.torch, self.dev = torch, dev
        self.enc, self.wdesc = _load_encoder(dev)
        mine = self.SEEDS[rank::world] or self.SEEDS[:1]
        imgs = [synth.synth_card(self.H, self.W, 500, 150, s) for s in mine]
        self.host = [x.contiguous().pin_memory() for x in imgs]
        self.dev_imgs = [x.to(dev) for x in imgs]
        # the single-image graph of the latency figure; PIPE_BATCH > 1 (--kernels-only --batch-graph) makes
        # it the throughput form's batch graph, for launch lists of that form
        self.pipe = pipeline.EncodeRender(self.enc, self.PIPE_BATCH, self.H, self.W, dev)
        self.stage_src = self.dev_imgs if self.PIPE_BATCH == 1 else self._batches(self.dev_imgs, n=self.PIPE_BATCH)
        self.i = 0

    def capture(self, profile=False):
        self.pipe.x.copy_(self.stage_src[0])
        self.pipe.capture(profile)

    def stage(self):
        """Put the next image into the pipeline's input buffer (outside the timed events)."""
        self.pipe.x.copy_(self.stage_src[self.i % len(self.stage_src)], non_blocking=True)
        self.i += 1

    def step(self):
        return self.pipe.replay()

    DEPTH = 3  # batches in flight (graph instances on their own streams)
    BATCH = 4  # images per graph replay in the throughput and e2e forms (one step = one batch)
    PIPE_BATCH = 1

    def _batches(self, cards, pin=False, n=None):
        """This rank's cards stacked into [n,3,H,W] batches (n = BATCH by default), every card used (cycled
        when a rank holds fewer than n)."""
        torch, B = self.torch, n or self.BATCH
        nb = max(1, len(cards) // B)
        out = [torch.stack([cards[(j * B + t) % len(cards)][0] for t in range(B)]) for j in range(nb)]
        return [x.contiguous().pin_memory() for x in out] if pin else out

    def _stream(self):
        from gaussian_2d_splat_encoder_b200 import pipeline

        if not hasattr(self, "stream"):
            self.stream = pipeline.EncodeRenderStream(self.enc, self.H, self.W, self.dev, depth=self.DEPTH,
                                                      batch=self.BATCH).capture()
            self.dev_batches = self._batches(self.dev_imgs)
        return self.stream

    def time_pipelined(self, K, warmup):
        """Whole-job throughput: K device-resident batches of BATCH cards (cycling through all of this
        rank's cards, 453 MB for 64, more than L2) through EncodeRenderStream with DEPTH batches in
        flight; CUDA events on the current stream around the K submits.  Returns the elapsed ms."""
        torch = self.torch
        st = self._stream()
        nb = len(self.dev_batches)
        st.start_after()
        for i in range(warmup):
            st.submit(self.dev_batches[i % nb])
        st.wait_into()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        st.start_after()
        for i in range(K):
            st.submit(self.dev_batches[(self.i + i) % nb])
        st.wait_into()
        b.record()
        torch.cuda.synchronize()
        self.i += K
        return a.elapsed_time(b)

    def e2e_buffers(self):
        """The streaming form of the public pipeline (EncodeRenderStream, DEPTH graph instances of BATCH
        images), pinned input batches and DEPTH pinned output batches."""
        self._stream()
        self.host_batches = self._batches(self.host, pin=True)
        return [self.torch.empty(self.BATCH, 3, self.H, self.W).pin_memory() for _ in range(self.DEPTH)]

    def e2e_begin(self):
        self.stream.start_after()

    def e2e_step(self, bufs):
        # H2D of this batch from pinned memory, encode + render, D2H of its reconstructions; the copies of
        # neighbouring batches overlap the kernels, up to DEPTH batches are in flight
        self.stream.submit(self.host_batches[self.i % len(self.host_batches)], bufs[self.i % len(bufs)])
        self.i += 1

    def e2e_end(self):
        self.stream.wait_into()

    def io_bytes(self):
        return self.BATCH * 3 * self.H * self.W * 4, self.BATCH * 3 * self.H * self.W * 4

    @classmethod
    def describe(cls, wdesc):
        """The workload both arms run (the reference arm's line carries the same keys)."""
        return {"workload": "configs 2/3: 768x768 test cards (seeds 100-163), EfficientGaussianEncoder forward + "
                            "render_alpha_octave(odds) of its splats, inference",
                "images_per_step_per_gpu": 1, "encoder_weights": wdesc, "H": cls.H, "W": cls.W,
                "splats_per_image": (cls.H // 8) ** 2 * 2 + (cls.H // 4) ** 2 * 2}

    def config(self):
        return {**self.describe(self.wdesc),
                "implementation": "bf16 tcgen05 encoder + fp32 render, one CUDA graph per batch",
                "images_per_step_per_gpu": self.BATCH,
                "images_in_flight": self.DEPTH * self.BATCH,
                "value_api": f"pipeline.EncodeRenderStream.submit(device batch of {self.BATCH}): one graph replay "
                             f"per batch, {self.DEPTH} graph instances on their own streams; every card of this "
                             "rank (64 x 7.1 MB at N=1) cycled, device-resident",
                "e2e_api": "pipeline.EncodeRenderStream.submit(pinned host batch, pinned host output): H2D -> "
                           f"encode+render graph -> D2H of the reconstructions, per batch of {self.BATCH}, "
                           f"{self.DEPTH} batches in flight, copies overlapped with the kernels",
                "latency_api": "pipeline.EncodeRender (batch 1): one graph replay per image",
                "l2": "inputs larger than L2 (the cycled cards, 453 MB at N=1) for value; the single-image "
                      "latency figure flushes L2 (256 MB write) between its timed steps"}

    @classmethod
    def cpu_inputs(cls):
        import torch

        from gaussian_2d_splat_encoder_b200 import synth

        sys.path.insert(0, str(ROOT / "tests"))
        from enc_util import GOLDEN_CFG

        m, desc = _load_encoder()
        return dict(sd=m.state_dict(), cfg=GOLDEN_CFG, x=synth.synth_card(cls.H, cls.W, 500, 150, cls.SEEDS[0]),
                    desc=desc, torch=torch)

    @classmethod
    def cpu_step(cls, O, s):
        from oracle import encoder_oracle as E

        o = E.encode(s["sd"], s["cfg"], s["x"])
        f = {k: (v.numpy() if v is not None else None) for k, v in o.items() if hasattr(v, "numpy") or v is None}
        O.render_alpha_octave(f["mu"], f["log_scale"], f["color"], f["opacity"], f["bg"], cls.H, cls.W,
                              theta=f["theta"], odds=True)


class RenderWorkload:
    """Config 1: render_alpha_octave(odds) forward + L2 backward of one 768^2 image, 92,160 splats."""

    name = "render"
    metric, unit, scaling = METRIC, "images/s", "weak"
    H = W = 768
    N = 92160

    def __init__(self, dev, rank=0, world=1):
        import torch

        from gaussian_2d_splat_encoder_b200 import pipeline, synth

        self.torch, self.dev = torch, dev
        s = synth.synth_splats_cfg1(self.N, self.H, self.W, seed=1)
        self.host = {k: v.contiguous().pin_memory() for k, v in s.items()}
        self.keys = ("mu", "log_scale", "color", "opacity", "bg", "theta")
        self.dev_in = {k: v.to(dev) for k, v in s.items()}
        self.pipe = pipeline.RenderFitStep(self.N, self.H, self.W, dev)

    def capture(self, profile=False):
        self.stage()
        self.pipe.capture(profile)

    def stage(self):
        self.pipe.load(*[self.dev_in[k] for k in self.keys], self.dev_in["target"])

    def step(self):
        return self.pipe.replay()

    def e2e_buffers(self):
        torch = self.torch
        bufs = [torch.empty(self.host[k].shape, dtype=torch.float32).pin_memory() for k in self.keys]
        bufs.append(torch.empty(1).pin_memory())
        return bufs

    def e2e_step(self, out_bufs):
        """Host (pinned) -> device copy of the step's inputs, the step, device -> host of loss + grads."""
        self.pipe.load(*[self.host[k] for k in self.keys], self.host["target"])
        loss, grads = self.pipe.replay()
        for o, g in zip(out_bufs, grads):
            o.copy_(g, non_blocking=True)
        out_bufs[-1].copy_(loss.detach().reshape(1), non_blocking=True)

    def io_bytes(self):
        h2d = sum(self.host[k].numel() * 4 for k in self.keys) + self.host["target"].numel() * 4
        d2h = sum(self.host[k].numel() * 4 for k in self.keys) + 4
        return h2d, d2h

    @classmethod
    def describe(cls, wdesc=None):
        return {"workload": "config 1: render_alpha_octave(odds=True) fwd + L2 bwd, 768x768, 92,160 splats (seed 1)",
                "images_per_step_per_gpu": 1, "H": cls.H, "W": cls.W, "splats": cls.N}

    def config(self):
        return {**self.describe(), "l2": "flushed between timed steps (256 MB write, outside the timed events)"}

    @classmethod
    def cpu_inputs(cls):
        from gaussian_2d_splat_encoder_b200 import synth

        return {k: v.numpy() for k, v in synth.synth_splats_cfg1(cls.N, cls.H, cls.W, seed=1).items()}

    @classmethod
    def cpu_step(cls, O, s):
        """One step of the reference's algorithm on the host: forward, L2 loss, backward (forward run once)."""
        O.render_alpha_octave_l2(s["mu"], s["log_scale"], s["color"], s["opacity"], s["bg"], cls.H, cls.W,
                                 s["target"], theta=s["theta"], odds=True)


def time_points(torch, dev, N=92160, P=3000, H=768, W=768, reps=20):
    """render_alpha_subsampled (render.py:68-87) forward + backward of sum(out * g): config-1 splats at
    P = 3000 sampled pixels (the released checkpoint's training n_pixels), eager calls timed with CUDA
    events.  Returns (ms per fwd+bwd, pixel-pairs per call)."""
    from gaussian_2d_splat_encoder_b200 import synth
    from gaussian_2d_splat_encoder_b200.render import render_alpha_subsampled

    s = synth.synth_splats_cfg1(N, H, W, seed=1)
    L = [s[k].to(dev).requires_grad_(True) for k in ("mu", "log_scale", "color", "opacity", "bg", "theta")]
    g = torch.Generator(device=dev).manual_seed(7)
    idx = torch.randint(0, H * W, (1, P), device=dev, generator=g)
    gout = torch.randn(1, 3, P, device=dev, generator=g)

    def one():
        out, _ = render_alpha_subsampled(*L[:5], H, W, theta=L[5], pixel_indices=idx)
        return torch.autograd.grad(out, L, grad_outputs=gout)

    for _ in range(3):
        one()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        one()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps, N * P


class FitWorkload:
    """Config 4: fitting loop on one 2048x2048 card (seed 4) with 655,360 splats initialised by the encoder.
    Rank r renders native rows [r*H/R, (r+1)*H/R) (render_alpha_octave row_band), the L2 loss is normalised
    by the global pixel count, the splat-parameter gradients (9 floats per splat + bg) are summed and split
    across ranks with one NCCL reduce-scatter, each rank runs the fused Adam step (lr 1e-2) on its 1/R of
    the parameters, and one all-gather returns the full parameters (shard.ShardedAdam).  One step = one CUDA
    graph replay (render fwd + bwd + reduce-scatter + Adam + all-gather)."""

    name = "fit"
    metric, unit, scaling = FIT_METRIC, "steps/s", "strong"
    H = W = 2048
    KEYS = ("mu", "log_scale", "color", "opacity", "bg", "theta")

    def __init__(self, dev, rank=0, world=1):
        import torch
        import torch.distributed as dist

        from gaussian_2d_splat_encoder_b200 import synth

        self.torch, self.dev, self.rank, self.world = torch, dev, rank, world
        self.dist = dist if world > 1 else None
        enc, self.wdesc = _load_encoder(dev)
        img = synth.card_for_config(4).to(dev)
        with torch.inference_mode():
            o = enc(img)
        self.keys = ("mu", "log_scale", "color", "opacity", "bg", "theta")
        self.init = {k: o[k].clone() for k in self.keys}
        self.leaves = [self.init[k].clone().requires_grad_(True) for k in self.keys]
        self.target = img.clone()
        self.N = self.init["mu"].shape[1]
        from gaussian_2d_splat_encoder_b200 import shard

        self.band = shard.row_bands(self.H, world)[rank]
        self.opt = shard.ShardedAdam(self.leaves, lr=1e-2)
        self.graph = None

        class _P:  # launches_per_replay holder, like the pipelines
            pass

        self.pipe = _P()

    def _body(self):
        from gaussian_2d_splat_encoder_b200 import pipeline

        L = self.leaves
        loss, grads = pipeline.render_l2_grads(L, self.target, self.H, self.W, True, self.band)
        self.opt.step(grads)
        return loss

    def capture(self, profile=False):
        torch = self.torch
        from gaussian_2d_splat_encoder_b200 import _lib
        from gaussian_2d_splat_encoder_b200 import render_triton as rt

        self.rt = rt
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self._body()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        L = _lib.load()
        if profile:
            L.gs_profile_collect2(None, None, 0)
            L.gs_profile_enable(1)
        n0 = L.gs_kernel_launches()
        with torch.cuda.graph(self.graph):
            self.loss = self._body()
        self.pipe.launches_per_replay = int(L.gs_kernel_launches() - n0)
        self.pipe.graph = self.graph
        if profile:
            L.gs_profile_enable(0)

    def stage(self):
        pass

    def step(self):
        self.graph.replay()
        return self.loss

    def e2e_buffers(self):
        return self.torch.empty(1).pin_memory()

    def e2e_step(self, buf):
        self.graph.replay()
        buf.copy_(self.loss.detach().reshape(1), non_blocking=True)

    def io_bytes(self):
        return 0, 4

    @classmethod
    def describe(cls, wdesc, N=655360):
        return {"workload": "config 4: 2048x2048 card (seed 4), 655,360 encoder-initialised splats, "
                            "render_alpha_octave(odds) fwd + L2 bwd + Adam lr 1e-2 per step",
                "splats": N, "H": cls.H, "W": cls.W, "encoder_weights": wdesc}

    def config(self):
        return {**self.describe(self.wdesc, self.N),
                "implementation": "render fwd+bwd on a native-row band per rank, NCCL reduce-scatter of the splat "
                                  "gradients, fused Adam; one CUDA graph per step",
                "band_rows": list(self.band),
                "l2": "flushed between timed steps (256 MB write, outside the timed events)"}

    @classmethod
    def cpu_inputs(cls):
        """Splats from the fp32 encoder oracle on the config-4 card, zeroed Adam moments."""
        import numpy as np

        from gaussian_2d_splat_encoder_b200 import synth
        from oracle import encoder_oracle as E

        sys.path.insert(0, str(ROOT / "tests"))
        from enc_util import GOLDEN_CFG

        m, desc = _load_encoder()
        img = synth.card_for_config(4)
        o = E.encode(m.state_dict(), GOLDEN_CFG, img)
        p = {k: np.ascontiguousarray(o[k].detach().numpy(), dtype=np.float32) for k in cls.KEYS}
        return dict(p=p, m={k: np.zeros_like(v) for k, v in p.items()}, v={k: np.zeros_like(v) for k, v in p.items()},
                    t=0, target=np.ascontiguousarray(img.numpy(), dtype=np.float32), desc=desc)

    @classmethod
    def cpu_step(cls, O, s):
        """One fitting step on the host: render forward, mse loss, backward, Adam (lr 1e-2, betas
        (0.9, 0.999), eps 1e-8: torch.optim.Adam's update) on every render input."""
        import numpy as np

        p = s["p"]
        _, _, _, g = O.render_alpha_octave_l2(p["mu"], p["log_scale"], p["color"], p["opacity"], p["bg"], cls.H,
                                              cls.W, s["target"], theta=p["theta"], odds=True)
        s["t"] += 1
        b1, b2, lr, eps = 0.9, 0.999, 1e-2, 1e-8
        c1, c2 = 1.0 - b1 ** s["t"], 1.0 - b2 ** s["t"]
        for k in cls.KEYS:
            m, v = s["m"][k], s["v"][k]
            m *= b1
            m += (1.0 - b1) * g[k]
            v *= b2
            v += (1.0 - b2) * g[k] * g[k]
            p[k] -= (lr / c1) * m / (np.sqrt(v / c2) + eps)

    def release(self):
        self.graph = None
        self.pipe.graph = None


WORKLOADS = {"encode_render": EncodeRenderWorkload, "render": RenderWorkload, "fit": FitWorkload}


# ------------------------------------------------------------------------------------------ CPU side
def cpu_baseline(workload_cls, steps: int, budget_s: float = 20.0, warmup: int = 1, warmup_budget_s: float = 60.0):
    """The reference's algorithm on the host cores (torch-CPU fp32 encoder + C oracle renderer, all
    threads): `warmup` untimed steps, then up to `steps` timed whole steps while the timed total stays
    under `budget_s` (at least one).  Returns (the cpu_baseline dict, the inputs' weight description)."""
    import torch

    from oracle import oracle as O

    O.build()
    # every host thread, whatever OMP_NUM_THREADS a launcher set (torchrun sets 1 per rank)
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    O.set_threads(n)
    s = workload_cls.cpu_inputs()
    t_w = time.perf_counter()
    nw = 0
    while nw < warmup and (nw == 0 or time.perf_counter() - t_w < warmup_budget_s):
        workload_cls.cpu_step(O, s)
        nw += 1
    times = []
    t_all = time.perf_counter()
    for _ in range(max(1, steps)):
        t0 = time.perf_counter()
        workload_cls.cpu_step(O, s)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_all > budget_s:
            break
    per = statistics.mean(times)
    res = workload_cls.H
    what = {"encode_render": "encode + render steps (one image each)", "render": "render fwd+bwd steps (one image each)",
            "fit": "fitting steps (render fwd + L2 bwd + Adam)"}[workload_cls.name]
    parts = (f"torch-CPU fp32 encoder ({torch.get_num_threads()} threads) + " if workload_cls.name == "encode_render"
             else "") + f"C oracle renderer ({O.num_threads()} OpenMP threads)"
    r = {"value": 1.0 / per, "unit": workload_cls.unit, "cores": O.num_threads(), "kind": "port",
         "sample": f"{len(times)} timed {what} at {res}x{res} after {nw} untimed, on the host: {parts}; "
                   f"os.cpu_count()={os.cpu_count()}"}
    if len(times) < steps:
        r["sample"] += f"; {len(times)} of the {steps} requested steps fitted the {budget_s:.0f} s bound"
    return r, s.get("desc") if isinstance(s, dict) else None


# ------------------------------------------------------------------------------------------ GPU timing
def time_steps(torch, wl, K, flush):
    """K graph replays, each bracketed by CUDA events on the replay stream; the L2 flush and the
    staging of the step's input happen between the events."""
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    for i in range(K):
        flush.zero_()
        wl.stage()
        ev[i][0].record()
        wl.step()
        ev[i][1].record()
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in ev]


def count_pairs(torch, lib, dev, ins, H, W, row_band=None):
    """(tile, splat) pairs of one octave-odds render of `ins` (read back from the binning)."""
    from gaussian_2d_splat_encoder_b200 import _lib
    from gaussian_2d_splat_encoder_b200.render_triton import _desc

    keys = ("mu", "log_scale", "color", "opacity", "bg", "theta")
    f = [ins[k].detach().contiguous().float() for k in keys]
    B, N = f[0].shape[0], f[0].shape[1]
    d = _desc(mode=_lib.MODE_OCTAVE, B=B, N=N, C=3, H=H, W=W, TILE=8, odds=True, has_theta=True, cutoff=3.0,
              base_texels=8.0, max_octaves=6, max_pairs=-1, row_band=row_band)
    d.pair_capacity = lib.gs_render_pair_bound(C.byref(d))
    nb = lib.gs_render_workspace_size(C.byref(d), 0)
    ws = torch.empty(nb, dtype=torch.uint8, device=dev)
    out = torch.empty(B, 3, H, W, device=dev)
    _lib.check(lib.gs_render_fwd(C.byref(d), *[_lib.ptr(t) for t in f], _lib.ptr(out), _lib.ptr(ws), nb,
                                 _lib.stream_of(dev)))
    torch.cuda.synchronize()
    tot = C.c_int64(0)
    _lib.check(lib.gs_render_debug_bins(C.byref(d), _lib.ptr(ws), C.byref(tot), None, None, None, None, None))
    return int(tot.value)


def octave_tiles(H, W, tile=8, max_octaves=6):
    """Tiles of an octave render: sum over octaves o of the TILE grid of max(8, H>>o) x max(8, W>>o)."""
    n = 0
    for o in range(max_octaves + 1):
        h, w = max(8, H >> o), max(8, W >> o)
        n += -(-h // tile) * -(-w // tile)
    return n


def binning_roofline(stages, pairs, N, H, W, hbm_gbs):
    """Binning of one render against HBM: algorithmic bytes N*36 (splat parameters read) + N*4 (per-splat
    pair counts) + pairs*8 (sorted (tile, splat) written once) + (tiles+1)*4 (tile ranges), over the
    measured time of the binning stage (memset, k_preprocess, k_tile_scan, k_scatter of one render)."""
    t = stages.get("binning", {}).get("ms_per_replay", 0.0) * 1e-3
    if t <= 0 or not pairs:
        return None
    nt = octave_tiles(H, W)
    nbytes = N * 36 + N * 4 + pairs * 8 + (nt + 1) * 4
    gbs = nbytes / t / 1e9
    return {"bound": "hbm", "kernels": "memset + k_preprocess + k_tile_scan + k_scatter", "ms": t * 1e3,
            "algorithmic_bytes": nbytes, "tiles": nt, "achieved_gbs": gbs, "peak_gbs": hbm_gbs,
            "frac": gbs / hbm_gbs}


def compositing_rooflines(stages, pairs, f_mhz):
    """Config-1 compositing against its rooflines, by fixed per-pixel-pair counts (pixel-pairs = pairs x
    64): forward 3 SFU (exp, log, rcp) + 17 FP32 ops, backward 2 SFU + 40 FP32 ops; peaks 148 SMs x 16
    MUFU and x 128 FP32 lanes per clock at the SM clock sampled in the timed region.  frac = roofline
    time / measured time of the kernel (stage events, one launch per replay)."""
    pp = pairs * 64
    sfu = 148 * 16 * f_mhz * 1e6  # ops/s
    fp32 = 148 * 128 * f_mhz * 1e6
    out = {"workload": "config 1 (92,160 splats, 768^2, odds)", "pairs": pairs, "pixel_pairs": pp,
           "peak_sfu_ops_per_s": sfu, "peak_fp32_ops_per_s": fp32,
           "peak_source": f"148 SMs x 16 MUFU / 128 FP32 lanes x {f_mhz:.0f} MHz (sampled SM clock)"}
    for key, kern, n_sfu, n_fp32 in (("fields_fwd", "k_fields_w8 + k_fields_deep8 (odds)", 3, 17),
                                     ("fields_bwd", "k_fields_bwd<8,4,odds>", 2, 40)):
        t = stages.get(key, {}).get("ms_per_replay", 0.0) * 1e-3
        if t <= 0:
            continue
        t_sfu, t_fp32 = pp * n_sfu / sfu, pp * n_fp32 / fp32
        out[key] = {"kernel": kern, "bound": "sfu" if t_sfu >= t_fp32 else "fp32", "ms": t * 1e3,
                    "roofline_ms": max(t_sfu, t_fp32) * 1e3, "frac": max(t_sfu, t_fp32) / t,
                    "achieved_sfu_ops_per_s": pp * n_sfu / t, "achieved_fp32_ops_per_s": pp * n_fp32 / t}
    return out


def profile_stages(torch, lib, wl_cls, dev, flush, reps=20, rank=0, world=1):
    """Per-stage device time from CUDA events the library records on its own stream around each stage,
    captured as event nodes into a separate graph of the same step and read after every replay."""
    from gaussian_2d_splat_encoder_b200 import _lib

    wl = wl_cls(dev, rank, world)
    wl.capture(profile=True)
    acc = {}
    ms = (C.c_double * 16)()
    cnt = (C.c_int64 * 16)()
    for _ in range(reps):
        flush.zero_()
        wl.stage()
        wl.step()
        torch.cuda.synchronize()
        _lib.check(lib.gs_profile_collect2(ms, cnt, 1))
        for i, n in STAGE_NAMES.items():
            if cnt[i] > 0:
                a = acc.setdefault(n, [0.0, int(cnt[i])])
                a[0] += ms[i]
    lib.gs_profile_collect2(None, None, 0)
    if hasattr(wl, "release"):
        wl.release()
    return {n: {"ms_per_replay": v[0] / reps, "calls_per_replay": v[1]} for n, v in acc.items()}


def encode_render_pairs(torch, lib, enc, x):
    """(tile, splat) pairs of one encode+render call: [encoder's internal 384^2 coarse render, final 768^2
    render], read back from a workspace this function owns (gs_encode_render_debug_pairs)."""
    from gaussian_2d_splat_encoder_b200 import _lib
    from gaussian_2d_splat_encoder_b200.efficient_encoder import cuda_forward

    B, _, H, W = x.shape
    d = enc._desc(B, H, W)
    nb = int(lib.gs_encode_render_workspace_size(C.byref(d)))
    ws = torch.empty(nb, dtype=torch.uint8, device=x.device)
    with torch.inference_mode():
        cuda_forward(enc, x, False, True, workspace=ws)
    torch.cuda.synchronize()
    pairs = (C.c_int64 * 2)()
    _lib.check(lib.gs_encode_render_debug_pairs(C.byref(d), _lib.ptr(ws), pairs), "gs_encode_render_debug_pairs")
    return int(pairs[0]), int(pairs[1])


def fields_fwd_roofline(stages, pairs_coarse, pairs_final, f_mhz, traffic=None):
    """k_fields_fwd of one encode+render step (the internal 384^2 coarse render + the final 768^2 render)
    against the SFU roofline: 3 SFU ops (exp, log, rcp) per pixel-pair in odds mode, pixel-pairs = pairs x
    64 (TILE 8), over the two launches' device time (stage events).  Peak: 148 SMs x 16 MUFU results per
    clock at the SM clock sampled during the timed region."""
    tc = stages.get("enc_fields_fwd", {}).get("ms_per_replay", 0.0)
    tf = stages.get("fields_fwd", {}).get("ms_per_replay", 0.0)
    if tc <= 0 or tf <= 0:
        return {"unavailable": "no stage times for the field kernels"}
    sfu = 148 * 16 * f_mhz * 1e6
    pp = (pairs_coarse + pairs_final) * 64
    t = (tc + tf) * 1e-3
    ach = 3.0 * pp / t
    per = {}
    for name, pr, tm in (("coarse_384", pairs_coarse, tc), ("final_768", pairs_final, tf)):
        ppr = pr * 64
        per[name] = {"pairs": pr, "pixel_pairs": ppr, "ms": tm, "roofline_ms": 3.0 * ppr / sfu * 1e3,
                     "frac": (3.0 * ppr / sfu) / (tm * 1e-3)}
    return {"bound": "sfu", "kernel": "k_fields_deep8 + k_fields_w8 (odds; coarse 384^2 render + final 768^2 render)",
            "achieved": ach / 1e12, "peak": sfu / 1e12, "unit": "T SFU-op/s", "frac": ach / sfu,
            "traffic": traffic, "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum, both launches of "
                                                   "one step (profiles/fields_fwd_encode_render_768.md)"
                                                   if traffic else None),
            "units_per_step": pp, "unit_name": "pixel-pair", "ops_per_unit": 3, "launches_per_step": 2,
            "ms_per_step": tc + tf, "per_render": per,
            "peak_source": f"148 SMs x 16 MUFU x {f_mhz:.0f} MHz (median SM clock sampled in the timed region)"}


def reference_triton_leg(torch, dev, H=768, W=768, warmup=5, runs=30):
    """The reference's own GPU path on this B200 (the denominator of the target's >= 50x): the unmodified
    reference package from baseline/_ref, EfficientGaussianEncoder forward + render_alpha_octave(odds) of
    its splats, timed with CUDA events per call after `warmup` calls (examples/encode_and_render.py:75-89
    of the reference, with the final render included), one config-3 card (seed 100), inference."""
    ref_root = ROOT / "baseline" / "_ref"
    if not (ref_root / "gaussian_splat_encoder" / "render_triton.py").exists():
        return {"unavailable": "reference package not present under baseline/_ref"}
    sys.path.insert(0, str(ref_root))
    try:
        import triton

        from gaussian_splat_encoder.efficient_encoder import EfficientGaussianEncoder as RefEnc
        from gaussian_splat_encoder.render_triton import render_alpha_octave as ref_render
    except Exception as ex:  # noqa: BLE001
        return {"unavailable": f"reference import failed: {type(ex).__name__}: {ex}"}
    finally:
        sys.path.remove(str(ref_root))
    from gaussian_2d_splat_encoder_b200 import synth

    sys.path.insert(0, str(ROOT / "tests"))
    from enc_util import GOLDEN_CFG, load_golden

    enc = load_golden(RefEnc)
    desc = "released checkpoint encoder_golden_d256.pt"
    if enc is None:
        torch.manual_seed(0)
        enc = RefEnc(**GOLDEN_CFG).eval()
        desc = "reference architecture, random init (torch.manual_seed(0))"
    enc = enc.to(dev)
    x = synth.synth_card(H, W, 500, 150, EncodeRenderWorkload.SEEDS[0]).to(dev)

    def one():
        with torch.no_grad():
            o = enc(x)
            return ref_render(o["mu"], o["log_scale"], o["color"], o["opacity"], o["bg"], H, W, theta=o["theta"],
                              odds=bool(getattr(enc, "odds", True)))

    t0 = time.perf_counter()
    for _ in range(warmup):
        one()
    torch.cuda.synchronize()
    t_warm = time.perf_counter() - t0
    ms = []
    for _ in range(runs):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        one()
        b.record()
        torch.cuda.synchronize()
        ms.append(a.elapsed_time(b))
    ms.sort()
    med = statistics.median(ms)
    # the same calls back to back (no synchronisation between images but the reference's own), one pair
    # of events around all of them: its whole-job throughput
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(runs):
        one()
    b.record()
    torch.cuda.synchronize()
    b2b = a.elapsed_time(b) / runs
    # the same path on batches of EncodeRenderWorkload.BATCH cards (our throughput form's batch), back to
    # back: its per-image cost when it, too, is given several images per call
    nb = EncodeRenderWorkload.BATCH
    xb = torch.stack([synth.synth_card(H, W, 500, 150, s)[0] for s in EncodeRenderWorkload.SEEDS[:nb]]).to(dev)

    def batch():
        with torch.no_grad():
            o = enc(xb)
            return ref_render(o["mu"], o["log_scale"], o["color"], o["opacity"], o["bg"], H, W, theta=o["theta"],
                              odds=bool(getattr(enc, "odds", True)))

    try:
        for _ in range(2):
            batch()
        a.record()
        for _ in range(max(1, runs // nb)):
            batch()
        b.record()
        torch.cuda.synchronize()
        bat = a.elapsed_time(b) / (max(1, runs // nb) * nb)
    except Exception:  # noqa: BLE001  (a batch the reference does not take: single images only)
        bat = float("inf")
    return {"images_per_s": 1000.0 / min(med, b2b, bat), "images_per_s_per_image_events": 1000.0 / med,
            "images_per_s_back_to_back": 1000.0 / b2b,
            f"images_per_s_batch{nb}": (1000.0 / bat) if bat != float("inf") else None,
            "ms_median": med, "ms_p10": ms[len(ms) // 10],
            "ms_p90": ms[(9 * len(ms)) // 10], "warmup": warmup, "runs": runs, "warmup_s_incl_jit": t_warm,
            "what": "unmodified reference (baseline/_ref/gaussian_splat_encoder): EfficientGaussianEncoder forward "
                    "(fp32 torch convs + its Triton 384^2 coarse render) + render_alpha_octave(odds=True) at 768^2, "
                    "torch.no_grad, no L2 flush; images_per_s = the best of CUDA events per image (median), the same "
                    "calls back to back (its host synchronisations inside _build_tiles stay) and batches of "
                    f"{nb} cards back to back",
            "encoder_weights": desc, "torch": torch.__version__, "triton": triton.__version__}


def fit_leg(torch, lib, dev, flush, rank, world, K=20, warmup=3, max_over_ranks=None, barrier=None):
    """Config 4 at this N (tile-row bands, NCCL reduce-scatter + all-gather around a sharded Adam per step):
    steps/s as the max over ranks of K graph replays, the field backward's roofline, and the two
    collectives alone."""
    wl = FitWorkload(dev, rank, world)
    wl.capture()
    for _ in range(warmup):
        wl.step()
    barrier()
    ms = time_steps(torch, wl, K, flush)
    tot = max_over_ranks(sum(ms))
    launches = wl.pipe.launches_per_replay
    band = list(wl.band)
    pairs = count_pairs(torch, lib, dev, {k: wl.init[k] for k in wl.keys}, wl.H, wl.W, wl.band)
    ar = None
    if world > 1:
        import torch.distributed as dist

        o = wl.opt

        def coll():
            dist.reduce_scatter_tensor(o.gshard, o.flat_g)
            dist.all_gather_into_tensor(o.flat_p, o.param.data)

        for _ in range(3):
            coll()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(K):
            coll()
        b.record()
        torch.cuda.synchronize()
        ar = {"ms": max_over_ranks(a.elapsed_time(b) / K), "bytes": o.flat_g.numel() * 4,
              "what": "NCCL reduce-scatter of the flattened splat gradients + all-gather of the updated "
                      "parameter shards, alone, eager, max over ranks"}
    wl.release()
    barrier()
    stages = profile_stages(torch, lib, FitWorkload, dev, flush, rank=rank, world=world)
    return {"metric": FIT_METRIC, "value": K / (tot / 1000.0), "unit": "steps/s", "ms_per_step": tot / K,
            "steps": K, "warmup": warmup, "band_rows_rank0": band, "pairs_rank0_band": pairs,
            "gpu_launches_per_step": launches, "stages_ms": stages, "allreduce": ar,
            "workload": FitWorkload.describe(wl.wdesc, wl.N)["workload"], "scaling": "strong"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="encode_render")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-fit", action="store_true", help="skip the config-4 sub-object of the default line")
    ap.add_argument("--no-reference-triton", action="store_true",
                    help="skip timing the reference's own GPU path (default line, N = 1)")
    ap.add_argument("--batch", type=int, default=EncodeRenderWorkload.BATCH,
                    help="images per graph replay in the throughput and e2e forms")
    ap.add_argument("--depth", type=int, default=EncodeRenderWorkload.DEPTH,
                    help="batches in flight in the throughput (value) and e2e measurements of encode_render")
    ap.add_argument("--batch-graph", action="store_true",
                    help="with --kernels-only: replay the throughput form's batch graph (--batch images)")
    ap.add_argument("--kernels-only", action="store_true",
                    help="warm-up + K graph replays and nothing else (for ncu launch lists)")
    args = ap.parse_args()
    W = max(3, args.warmup)
    K = max(1, args.steps)
    EncodeRenderWorkload.DEPTH = max(1, args.depth)
    EncodeRenderWorkload.BATCH = max(1, args.batch)
    if args.kernels_only and args.batch_graph:
        EncodeRenderWorkload.PIPE_BATCH = EncodeRenderWorkload.BATCH
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    wcls = WORKLOADS[args.workload]

    if args.impl == "reference":
        if rank != 0:
            return
        r, wdesc = cpu_baseline(wcls, K, budget_s=150.0, warmup=W)
        line = {"metric": wcls.metric, "value": r["value"], "unit": wcls.unit, "n_gpus": args.gpus, "steps": K,
                "warmup": W, "ms_per_step": 1000.0 / r["value"], "higher_is_better": True, "scaling": wcls.scaling,
                "vs_baseline": None, "dtype": "fp32", "data": "synthetic", "impl": "reference",
                "config": {**wcls.describe(wdesc), "implementation": "host CPU: the reference's algorithm restated "
                           "(oracle/), all host threads", "parallelism": "rank 0 only (host cores)"},
                "cpu_baseline": r,
                "e2e": {"value": r["value"], "unit": wcls.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist

    from gaussian_2d_splat_encoder_b200 import _lib

    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lib = _lib.load()
    if args.kernels_only:
        # lean process for ncu (it saves and restores device memory between passes): one input image and
        # no L2-flush buffer (ncu flushes caches itself)
        EncodeRenderWorkload.SEEDS = EncodeRenderWorkload.SEEDS[:1]
    wl = wcls(dev, rank, world)
    flush = torch.empty(L2_FLUSH_BYTES // 4 if not args.kernels_only else 1024, dtype=torch.float32, device=dev)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    wl.capture()
    per_replay = wl.pipe.launches_per_replay  # our kernels (memsets included) in one graph replay
    for _ in range(W):
        wl.stage()
        wl.step()
    barrier()
    if args.kernels_only:
        time_steps(torch, wl, K, flush)
        if hasattr(wl, "release"):
            wl.release()
        if world > 1:
            dist.destroy_process_group()
        return
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    idx = int(vis.split(",")[local]) if vis else local
    try:
        import uuid as _uuid

        uuid = str(_uuid.UUID(bytes=bytes(torch.cuda.get_device_properties(dev).uuid.bytes)))
    except Exception:
        uuid = None
    pipelined = hasattr(wl, "time_pipelined")
    with ClockSampler(idx, uuid) as clk:
        with clk.window():
            step_ms = time_steps(torch, wl, K, flush)
            if pipelined:
                barrier()
                thr_ms = wl.time_pipelined(K, W)
    # our kernels in the value's timed region (one replay per step of the pipelined graphs)
    launches = (wl.stream.slots[0].launches_per_replay if pipelined else per_replay) * K
    lat_ms = max_over_ranks(sum(step_ms))
    # value: whole-job throughput (images in flight where the workload pipelines them), max over ranks
    tot_ms = max_over_ranks(thr_ms) if pipelined else lat_ms
    barrier()

    # end-to-end through the public API with host buffers (H2D of inputs, D2H of the result inside)
    buf = wl.e2e_buffers()
    for _ in range(2):
        wl.e2e_step(buf)
    barrier()
    Ke = max(3, min(K, 50))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if hasattr(wl, "e2e_end"):
        wl.e2e_end()
    e0.record()
    if hasattr(wl, "e2e_begin"):
        wl.e2e_begin()
    for _ in range(Ke):
        wl.e2e_step(buf)
    if hasattr(wl, "e2e_end"):
        wl.e2e_end()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))

    # per-stage device times (separate profiled graph) and the secondary config-1 metric
    stages = profile_stages(torch, lib, wcls, dev, flush, rank=rank, world=world)
    sec = None
    if wcls is EncodeRenderWorkload:
        rw = RenderWorkload(dev)
        rw.capture()
        for _ in range(3):
            rw.stage()
            rw.step()
        rms = time_steps(torch, rw, 50, flush)
        sec = {"render_fwd_bwd_ms_per_image": statistics.mean(rms),
               "stages_ms": profile_stages(torch, lib, RenderWorkload, dev, flush)}
        try:  # (tile, splat) pairs of the config-1 render, for its compositing rooflines
            sec["pairs"] = count_pairs(torch, lib, dev, rw.dev_in, rw.H, rw.W)
        except Exception as ex:
            sec["pairs"] = None
            sec["pairs_error"] = f"{type(ex).__name__}: {ex}"
        pms, ppairs = time_points(torch, dev)
        sec["points"] = {"workload": "render_alpha_subsampled fwd+bwd, 92,160 config-1 splats x 3,000 pixels",
                         "ms_per_step": pms, "pixel_pairs": ppairs,
                         "gpixel_pairs_per_s": ppairs / (pms * 1e-3) / 1e9}
    barrier()

    ips = getattr(wl, "BATCH", 1)  # images per step of the throughput and e2e forms
    images = K * world * (ips if pipelined else 1)
    value = images / (tot_ms / 1000.0)
    e2e_val = Ke * world * ips / (e2e_ms / 1000.0)
    h2d, d2h = wl.io_bytes()
    clocks = clk.summary()
    f_mhz = clocks["sm_mhz"] or 1965.0
    pk = peaks()
    line = {
        "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": tot_ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 encoder / fp32 render" if wcls is EncodeRenderWorkload else "fp32", "data": "synthetic",
        "config": {**wl.config(), "parallelism": (f"tile-row bands x{world}, NCCL reduce-scatter / all-gather of the splat "
                                                  "gradients per step" if wcls is FitWorkload else
                                                  f"dp{world} (image per GPU, no collective)")},
        "stages_ms": stages, "clocks": clocks, "gpu_launches": int(launches),
        "e2e": {"value": e2e_val, "unit": "images/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "peaks": pk,
    }
    if pipelined:
        line["latency"] = {"images_per_s": K * world / (lat_ms / 1000.0), "ms_per_image": lat_ms / K,
                           "what": "one image per step, one graph replay per step, each step timed alone with "
                                   "CUDA events, L2 flushed (256 MB write) between steps; max over ranks"}
    if wcls is EncodeRenderWorkload:
        # dominant kernel of the step: k_fields_fwd (both renders), SFU-bound
        try:
            pc, pf = encode_render_pairs(torch, lib, wl.enc, wl.dev_imgs[0])
            line["roofline"] = fields_fwd_roofline(stages, pc, pf, f_mhz, traffic=FIELDS_FWD_TRAFFIC)
        except Exception as ex:  # noqa: BLE001
            line["roofline"] = {"unavailable": f"{type(ex).__name__}: {ex}"}
        # secondary: the decoder convolution (tensor-bound, off the critical path): 2*M*N*K flops per launch
        M, N, Kd = (wl.H // 4) * (wl.W // 4), 128, 9 * 384
        t = stages.get("conv4_decoder", {}).get("ms_per_replay", 0.0)
        ach = 2.0 * M * N * Kd / (t * 1e-3) / 1e12 if t > 0 else None
        line["roofline_decoder"] = {"bound": "tensor", "kernel": "k_conv_tc (decoder 3x3 384->128 @192^2)",
                                    "achieved": ach, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                                    "frac": (ach / pk["bf16_tflops"]) if ach else None,
                                    "algorithmic_bytes": 2 * M * (256 + 128) + 2 * N * Kd + 2 * M * N,
                                    "flops_per_launch": 2.0 * M * N * Kd,
                                    "peak_source": f"MEASURED_PEAKS.json bf16_tflops (burst, {pk['source']})"}
        line["render_fwd_bwd_ms_per_image"] = sec["render_fwd_bwd_ms_per_image"] if sec else None
        line["render_stages_ms"] = sec["stages_ms"] if sec else None
        if sec:
            line["render_roofline"] = (compositing_rooflines(sec["stages_ms"], sec["pairs"], f_mhz) if sec["pairs"]
                                       else {"unavailable": sec.get("pairs_error", "no pair count")})
            if sec["pairs"]:
                line["render_roofline"]["binning"] = binning_roofline(sec["stages_ms"], sec["pairs"],
                                                                      RenderWorkload.N, RenderWorkload.H,
                                                                      RenderWorkload.W, pk["hbm_gbs"])
        line["points_fwd_bwd"] = sec["points"] if sec else None
    else:
        if wcls is RenderWorkload:
            line["render_fwd_bwd_ms_per_image"] = tot_ms / K
            pairs = count_pairs(torch, lib, dev, wl.dev_in, wl.H, wl.W)
        else:
            line.update(unit=wcls.unit, scaling=wcls.scaling, dtype="fp32", metric=wcls.metric)
            line["value"] = K / (tot_ms / 1000.0)
            line["e2e"]["value"] = Ke / (e2e_ms / 1000.0)
            line["e2e"]["unit"] = "steps/s"
            pairs = count_pairs(torch, lib, dev, {k: wl.init[k] for k in wl.keys}, wl.H, wl.W, wl.band)
        fw = stages.get("fields_bwd", {}).get("ms_per_replay", 0.0)
        pp = pairs * 64
        fp32_peak = 148 * 128 * f_mhz * 1e6 / 1e9
        ach = 40.0 * pp / (fw * 1e-3) / 1e9 if fw > 0 else None
        line["roofline"] = {"bound": "fp32", "kernel": "k_fields_bwd<8,4>", "achieved": ach, "peak": fp32_peak,
                            "unit": "Gop/s (FP32 lane-ops)", "frac": (ach / fp32_peak) if ach else None,
                            "traffic": None, "units_per_launch": pp, "ops_per_unit": 40, "pairs": pairs,
                            "peak_source": f"148 SMs x 128 FP32 lanes x {f_mhz:.0f} MHz (median SM clock sampled "
                                           "during the timed region)"}
    if wcls is EncodeRenderWorkload and not args.no_fit:
        # config 4 at this N: the one path with a collective (every rank takes part)
        fit = fit_leg(torch, lib, dev, flush, rank, world, max_over_ranks=max_over_ranks, barrier=barrier)
        fb = fit["stages_ms"].get("fields_bwd", {}).get("ms_per_replay", 0.0)
        fp32_peak = 148 * 128 * f_mhz * 1e6
        if fb > 0:
            fit["fields_bwd_roofline"] = {"bound": "fp32", "ops_per_pixel_pair": 40,
                                          "pixel_pairs_rank0": fit["pairs_rank0_band"] * 64,
                                          "frac": 40.0 * fit["pairs_rank0_band"] * 64 / fp32_peak / (fb * 1e-3)}
        line["fit"] = fit
    if wcls is EncodeRenderWorkload and world == 1 and not args.no_reference_triton:
        try:
            rt = reference_triton_leg(torch, dev)
        except Exception as ex:  # noqa: BLE001
            rt = {"unavailable": f"reference run failed: {type(ex).__name__}: {ex}"}
        if "images_per_s" in rt:
            rt["ours_over_reference"] = value / rt["images_per_s"]
            rt["ours_e2e_over_reference"] = e2e_val / rt["images_per_s"]
            if "latency" in line:
                rt["ours_latency_over_reference"] = line["latency"]["images_per_s"] / rt["images_per_s"]
            rt["target"] = ">= 50x (north_star)"
        line["reference_triton"] = rt
    if rank == 0 and world == 1 and not args.no_cpu_baseline:  # the host baseline is an N = 1 figure
        line["cpu_baseline"] = cpu_baseline(wcls, 3)[0]
    if rank == 0:
        print(json.dumps(line), flush=True)
    if hasattr(wl, "release"):
        wl.release()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
