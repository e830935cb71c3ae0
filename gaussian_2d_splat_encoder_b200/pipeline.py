"""CUDA-graph pipelines over the encode-and-render path.

Every kernel of the path is launched from host code (Python wrappers + the C ABI), which costs a few
microseconds of CPU per launch; at 768^2 the GPU work of one image is well under a millisecond, so an
eagerly launched step is bound by the host.  These classes capture a whole step once per input shape
into a CUDA graph and replay it: the same kernels, the same numerics, one launch.

* ``EncodeRender`` -- ``EfficientGaussianEncoder`` forward + ``render_alpha_octave`` of its splats
  (examples/encode_and_render.py:31-38 of the reference), inference.
* ``EncodeRenderStream`` -- the same for a stream of image batches, several in flight at once on their
  own streams, with the PCIe copies of neighbouring batches overlapped with the kernels.
* ``RenderFitStep`` -- ``render_alpha_octave`` forward + an L2 loss + the gradients of the six splat
  leaves (the fitting step of configs 1 and 4).

Outputs live in static buffers that the next call overwrites; clone them to keep them.
"""

from __future__ import annotations

import torch

from . import _lib
from .render_triton import render_alpha_octave


class EncodeRender:
    def __init__(self, encoder, batch: int, H: int, W: int, device=None, warmup: int = 2):
        self.enc = encoder
        if device is None:  # the module's parameters, or a PackedEncoder's device
            device = next(encoder.parameters()).device if hasattr(encoder, "parameters") else encoder.device
        self.dev = torch.device(device)
        self.shape = (batch, 3, H, W)
        self.x = torch.zeros(self.shape, device=self.dev)
        self.graph = None
        self.out = None
        self.rec = None
        self.warmup = warmup

    def _body(self):
        # one library call (gs_encode_render_fwd): the render reuses the encoder's coarse-render fields
        return self.enc.forward_and_render(self.x)

    def capture(self, profile: bool = False):
        """Warm up eagerly, then capture one step.  profile=True captures the library's stage events
        (gs_profile_enable) into the graph so every replay re-records them."""
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.inference_mode(), torch.cuda.stream(s):
            for _ in range(self.warmup):
                self._body()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        L = _lib.load()
        if profile:
            L.gs_profile_collect2(None, None, 0)
            L.gs_profile_enable(1)
        n0 = L.gs_kernel_launches()
        with torch.inference_mode(), torch.cuda.graph(self.graph):
            self.out, self.rec = self._body()
        self.launches_per_replay = int(L.gs_kernel_launches() - n0)
        if profile:
            L.gs_profile_enable(0)
        return self

    def __call__(self, image: torch.Tensor):
        """image [B,3,H,W] (device or pinned host memory) -> reconstruction [B,3,H,W] (static buffer).
        The encoder outputs of the same call are in ``self.out``."""
        if self.graph is None:
            self.capture()
        self.x.copy_(image, non_blocking=True)
        self.graph.replay()
        return self.rec

    def replay(self):
        self.graph.replay()
        return self.rec


class EncodeRenderStream:
    """Throughput form of ``EncodeRender`` for a stream of host images (config 3's image batches).

    ``depth`` graph instances, each with its own input, workspace and output buffers and its own compute
    stream, take batches of ``batch`` images in turn: up to ``depth * batch`` images are encoded and
    rendered at once (one image's latency-bound kernel chains -- binning, the small convolutions -- leave
    most SMs idle; a batch gives every launch ``batch`` images' work and the neighbouring batches fill
    what is left), and the host-to-device copy of the next batch and the device-to-host copy of a
    finished reconstruction run on their own streams, so PCIe traffic hides behind the kernels.
    ``submit(images, out)`` enqueues one batch (pinned host or device [batch,3,H,W]) and optionally its
    destination (pinned host [batch,3,H,W]); ``synchronize()`` waits for every submitted reconstruction."""

    def __init__(self, encoder, H: int, W: int, device=None, depth: int = 4, batch: int = 1):
        self.batch = batch
        self.slots = [EncodeRender(encoder, batch, H, W, device) for _ in range(depth)]
        dev = self.slots[0].dev
        self.dev = dev
        self.h2d, self.d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        self.comps = [torch.cuda.Stream(dev) for _ in range(depth)]
        mk = lambda: [torch.cuda.Event() for _ in range(depth)]  # noqa: E731
        self.ev_in, self.ev_done, self.ev_out = mk(), mk(), mk()
        self.used = [False] * depth
        self.n = 0

    def capture(self):
        for s in self.slots:
            s.capture()
        return self

    def submit(self, image: torch.Tensor, out: torch.Tensor | None = None):
        """Enqueue one batch of images.  A host batch (pinned) is copied in on the H2D stream; a device
        batch is copied into the slot's input buffer on the slot's own stream.  With `out` (pinned host) the
        reconstruction is copied out on the D2H stream; without it, it stays in the slot's static buffer,
        which is returned and stays valid until that slot's next batch (``depth`` submits later)."""
        k = self.n % len(self.slots)
        slot = self.slots[k]
        if slot.graph is None:
            slot.capture()
        comp = self.comps[k]
        if self.used[k]:
            comp.wait_event(self.ev_out[k])        # the slot's output buffer was copied out
        if image.is_cuda:
            with torch.cuda.stream(comp):
                slot.x.copy_(image, non_blocking=True)
        else:
            if self.used[k]:
                self.h2d.wait_event(self.ev_done[k])   # the slot's input buffer was read by its last replay
            with torch.cuda.stream(self.h2d):
                slot.x.copy_(image, non_blocking=True)
                self.ev_in[k].record(self.h2d)
            comp.wait_event(self.ev_in[k])
        with torch.cuda.stream(comp):
            slot.graph.replay()
            self.ev_done[k].record(comp)
        if out is not None:
            self.d2h.wait_event(self.ev_done[k])
            with torch.cuda.stream(self.d2h):
                out.copy_(slot.rec, non_blocking=True)
                self.ev_out[k].record(self.d2h)
        else:
            self.ev_out[k].record(comp)
        self.used[k] = True
        self.n += 1
        return slot.rec

    def wait_into(self, stream=None):
        """Make `stream` (default: the current stream) wait for every submitted image."""
        st = stream if stream is not None else torch.cuda.current_stream(self.dev)
        for k, u in enumerate(self.used):
            if u:
                st.wait_event(self.ev_out[k])

    def start_after(self, stream=None):
        """Order the pipeline's streams after the work already queued on `stream` (default: current)."""
        st = stream if stream is not None else torch.cuda.current_stream(self.dev)
        for s in (self.h2d, self.d2h, *self.comps):
            s.wait_stream(st)

    def synchronize(self):
        for s in (self.h2d, self.d2h, *self.comps):
            s.synchronize()


def render_l2_grads(leaves, target, H: int, W: int, odds: bool = True, row_band=None):
    """One fitting step's loss and gradients: render_alpha_octave forward, the fused L2 kernel
    (gs_l2_loss_grad: mse over the whole image, or a row band's share of it), and the render backward
    seeded with that gradient.  Returns (loss [1] device tensor, grads of the six leaves)."""
    L = leaves
    out = render_alpha_octave(L[0], L[1], L[2], L[3], L[4], H, W, theta=L[5], odds=odds, row_band=row_band)
    dev = out.device
    gout = torch.zeros_like(out) if row_band is not None else torch.empty_like(out)
    loss = torch.empty(1, device=dev)
    y0, y1 = row_band if row_band is not None else (0, H)
    planes = out.shape[0] * out.shape[1]
    tgt = target.contiguous().float()
    _lib.check(_lib.load().gs_l2_loss_grad(_lib.ptr(out), _lib.ptr(tgt), planes, H, W, y0, y1,
                                           1.0 / float(planes * H * W), _lib.ptr(gout), _lib.ptr(loss),
                                           _lib.stream_of(dev)), "gs_l2_loss_grad")
    grads = torch.autograd.grad(out, L, grad_outputs=gout)
    return loss, grads


class RenderFitStep:
    def __init__(self, N: int, H: int, W: int, device, batch: int = 1, odds: bool = True, warmup: int = 2):
        self.dev = torch.device(device)
        self.H, self.W, self.odds = H, W, odds
        self.leaves = [torch.zeros(batch, N, 2, device=self.dev), torch.zeros(batch, N, 2, device=self.dev),
                       torch.zeros(batch, N, 3, device=self.dev), torch.zeros(batch, N, device=self.dev),
                       torch.zeros(batch, 3, device=self.dev), torch.zeros(batch, N, device=self.dev)]
        for t in self.leaves:
            t.requires_grad_(True)
        self.target = torch.zeros(batch, 3, H, W, device=self.dev)
        self.graph = None
        self.warmup = warmup

    def load(self, mu, log_scale, color, opacity, bg, theta, target):
        with torch.no_grad():
            for dst, src in zip(self.leaves, (mu, log_scale, color, opacity, bg, theta)):
                dst.copy_(src, non_blocking=True)
            self.target.copy_(target, non_blocking=True)

    def _body(self):
        return render_l2_grads(self.leaves, self.target, self.H, self.W, self.odds)

    def capture(self, profile: bool = False):
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for _ in range(self.warmup):
                self._body()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        L = _lib.load()
        if profile:
            L.gs_profile_collect2(None, None, 0)
            L.gs_profile_enable(1)
        n0 = L.gs_kernel_launches()
        with torch.cuda.graph(self.graph):
            self.loss, self.grads = self._body()
        self.launches_per_replay = int(L.gs_kernel_launches() - n0)
        if profile:
            L.gs_profile_enable(0)
        return self

    def replay(self):
        if self.graph is None:
            self.capture()
        self.graph.replay()
        return self.loss, self.grads
