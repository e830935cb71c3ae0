"""Render entry points of the reference's ``render_triton`` module, backed by sm_100a CUDA kernels.

Drop-in for bigwolfeman/gaussian-2d-splat-encoder ``gaussian_splat_encoder/render_triton.py``: same
function names, arguments, defaults, output shapes and exceptions.  The module keeps its reference name
so callers only change the package import; nothing here uses Triton.  All work happens in
``libgsplat_b200.so`` (see include/gsplat_b200.h):

* ``render_alpha_octave``       render_triton.py:935-980   (GS_MODE_OCTAVE)
* ``render_alpha_full_triton``  render_triton.py:326-347   (cull=True: GS_MODE_CULL, cull=False: GS_MODE_EXACT)
* ``render_alpha_multires``     render_triton.py:879-922   (GS_MODE_MULTIRES)

Math (identical to the reference): a = min(o * exp(-maha/2), 1 - 1e-4); T = exp(sum log(1 - a));
fg = sum(w c) / max(sum w, 1e-8) with w = a (alpha) or a/(1-a) (odds); C = (1 - T) fg + T bg.  Each
call is differentiable w.r.t. mu, log_scale, color, opacity, bg and theta.
"""

from __future__ import annotations

import ctypes as _C

import torch

from . import _lib
from .params import activate_scale  # noqa: F401  (re-exported like the reference module)


class PairBudgetExceeded(RuntimeError):
    """A render would hold more (tile, splat) pairs for one image and group than ``max_pairs``
    (reference: render_triton.py:51-54).  Raised before the pair buffers are allocated."""


# Above this many pairs the host-side bound is replaced by an exact device count (one sync) before
# the workspace is sized, so a pathological bound never turns into a huge allocation.
_BOUND_SYNC_THRESHOLD = 1 << 26


def _desc(mode, B, N, C, H, W, TILE, odds, has_theta, cutoff, base_texels=8.0, max_octaves=6, n_coarse=-1,
          coarse_factor=8, max_pairs=-1, capacity=0, row_band=None):
    d = _lib.GsRenderDesc()
    d.mode, d.B, d.N, d.C, d.H, d.W = int(mode), int(B), int(N), int(C), int(H), int(W)
    d.tile, d.odds, d.has_theta = int(TILE), int(bool(odds)), int(bool(has_theta))
    d.max_octaves, d.n_coarse, d.coarse_factor = int(max_octaves), int(n_coarse), int(coarse_factor)
    d.cutoff, d.base_texels = float(cutoff), float(base_texels)
    d.max_pairs = -1 if max_pairs is None else int(max_pairs)
    d.pair_capacity = int(capacity)
    if row_band is not None:
        d.row_begin, d.row_end = int(row_band[0]), int(row_band[1])
    return d


def _f32(t):
    return None if t is None else t.detach().contiguous().float()


def _size_pairs(d, mu, ls, dev, H, W, N, TILE, cutoff):
    """Pair capacity for the workspace: the host bound when it is within budget, else the exact count
    (the reference's _build_tiles budget check, render_triton.py:378-385)."""
    L = _lib.load()
    bound = int(L.gs_render_pair_bound(C_ref(d)))
    if bound < 0:
        raise ValueError("invalid render arguments")
    per_image = bound // max(d.B, 1)
    need_exact = bound > _BOUND_SYNC_THRESHOLD or (d.max_pairs >= 0 and per_image > d.max_pairs)
    if not need_exact:
        return bound
    d0 = _lib.GsRenderDesc.from_buffer_copy(d)
    d0.pair_capacity = 1
    ws = torch.empty(int(L.gs_render_workspace_size(C_ref(d0), 0)), dtype=torch.uint8, device=dev)
    groups = (d.max_octaves + 1) if d.mode == _lib.MODE_OCTAVE else (2 if d.mode == _lib.MODE_MULTIRES else 1)
    counts = (C_int64 * (d.B * groups))()
    ng = C_int32(0)
    _lib.check(L.gs_render_count(C_ref(d0), _lib.ptr(mu), _lib.ptr(ls), _lib.ptr(ws), ws.numel(),
                                 counts, C_ref(ng), _lib.stream_of(dev)), "gs_render_count")
    c = list(counts)
    worst = max(c) if c else 0
    if d.max_pairs >= 0 and worst > d.max_pairs:
        raise PairBudgetExceeded(
            f"render: {worst} (tile,gaussian) pairs exceeds the {d.max_pairs} budget @ {H}x{W} TILE={TILE} "
            f"cutoff={cutoff} N={N}. Large splats bin into nearly every tile at this resolution; render them "
            f"through a low-resolution group instead. Refusing to allocate.")
    return max(sum(c), 1)


C_int64, C_int32 = _C.c_int64, _C.c_int32


def C_ref(x):
    return _C.byref(x)


class _Render(torch.autograd.Function):
    """One autograd node for a whole (batched, all-group) render; the workspace of the forward
    carries the binning and the field sums into the backward."""

    @staticmethod
    def forward(ctx, mu, log_scale, color, opacity, bg, theta, cfg):
        dev = _lib.require_cuda(mu, log_scale, color, opacity, bg, theta)
        mode, H, W, kw = cfg
        B, N, Cc = color.shape
        if mu.shape != (B, N, 2) or log_scale.shape != (B, N, 2) or opacity.shape != (B, N) or bg.shape[0] != B:
            raise ValueError("shape mismatch: mu/log_scale [B,N,2], color [B,N,C], opacity [B,N], bg [B,C]")
        if not 1 <= Cc <= 3:
            raise ValueError(f"colour channels of one render call must be 1..3, got {Cc}")
        f = [_f32(t) for t in (mu, log_scale, color, opacity, bg, theta)]
        has_th = theta is not None
        with torch.cuda.device(dev):
            d = _desc(mode, B, N, Cc, H, W, has_theta=has_th, **kw)
            L = _lib.load()
            if mode != _lib.MODE_EXACT:
                d.pair_capacity = _size_pairs(d, f[0], f[1], dev, H, W, N, kw["TILE"], kw["cutoff"])
            train = any(ctx.needs_input_grad[:6])
            nbytes = int(L.gs_render_workspace_size(C_ref(d), int(train)))
            if nbytes == 0:
                raise ValueError("invalid render arguments")
            ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            out = torch.empty((B, Cc, H, W), dtype=torch.float32, device=dev)
            _lib.check(L.gs_render_fwd(C_ref(d), *[_lib.ptr(t) for t in f], _lib.ptr(out), _lib.ptr(ws), nbytes,
                                       _lib.stream_of(dev)), "gs_render_fwd")
        ctx.desc = d
        ctx.ws = ws if train else None
        ctx.has_theta = has_th
        ctx.save_for_backward(*[t if t is not None else mu.new_zeros(0) for t in f])
        return out

    @staticmethod
    def backward(ctx, grad_out):
        mu, ls, col, op, bg, th = ctx.saved_tensors
        th = th if ctx.has_theta else None
        dev = mu.device
        g = grad_out.contiguous().float()
        grads = [torch.empty_like(mu), torch.empty_like(ls), torch.empty_like(col), torch.empty_like(op),
                 torch.empty_like(bg), torch.empty_like(th) if th is not None else None]
        with torch.cuda.device(dev):
            L = _lib.load()
            ws = ctx.ws
            _lib.check(L.gs_render_bwd(C_ref(ctx.desc), _lib.ptr(mu), _lib.ptr(ls), _lib.ptr(col), _lib.ptr(op),
                                       _lib.ptr(bg), _lib.ptr(th), _lib.ptr(g), *[_lib.ptr(x) for x in grads],
                                       _lib.ptr(ws), ws.numel(), _lib.stream_of(dev)), "gs_render_bwd")
        out = [gr if ctx.needs_input_grad[i] else None for i, gr in enumerate(grads)]
        return (*out, None)


def _render(mode, mu, log_scale, color, opacity, bg, H, W, theta, kw):
    cfg = (mode, int(H), int(W), kw)
    C = color.shape[-1]
    if C <= 3:
        return _Render.apply(mu, log_scale, color, opacity, bg, theta, cfg)
    # More than three channels (the reference's kernels take any C): the transmittance and the weight sum
    # do not depend on colour and every output channel composites on its own, so groups of at most three
    # channels render independently and concatenate exactly; autograd sums the shared leaves' gradients.
    return torch.cat([_Render.apply(mu, log_scale, color[..., c:c + 3], opacity, bg[:, c:c + 3], theta, cfg)
                      for c in range(0, C, 3)], dim=1)


def render_alpha_octave(mu, log_scale, color, opacity, bg, H, W, theta=None, cutoff=3.0, TILE=8,
                        base_texels=8.0, max_octaves=6, max_pairs=48_000_000, odds=False, row_band=None):
    """Memory-bounded differentiable render with scale-routed octave LOD (render_triton.py:935-980).

    Each splat renders at octave o = clamp(ceil(log2(max(sigma_px / base_texels, 1e-6))), 0, max_octaves)
    at resolution max(8, H >> o) x max(8, W >> o); the octaves' raw sums are bilinearly upsampled
    (align_corners=False), summed and composited once with bg.  Returns [B,C,H,W] float32.
    Raises PairBudgetExceeded when one image's octave would hold more than max_pairs pairs.

    row_band=(y0, y1) (an extension for tile-row sharding across GPUs) renders only native rows
    [y0, y1): only the splats whose footprint reaches those rows are binned, output rows outside the band
    are left unwritten, and the backward reads grad_out only inside the band, so the gradients are the
    band's partial sums (summing them over a partition of the rows gives the full gradient)."""
    if not 0 <= int(max_octaves) <= 7:
        raise ValueError("max_octaves must be in 0..7")
    kw = dict(TILE=TILE, odds=odds, cutoff=cutoff, base_texels=base_texels, max_octaves=max_octaves,
              max_pairs=max_pairs, row_band=row_band)
    return _render(_lib.MODE_OCTAVE, mu, log_scale, color, opacity, bg, H, W, theta, kw)


def render_alpha_full_triton(mu, log_scale, color, opacity, bg, H, W, theta=None, cull=False, TILE=8,
                             cutoff=3.0, odds=False):
    """Single-resolution render (render_triton.py:326-347).  cull=True bins splats into TILE x TILE tiles by
    their cutoff*max-sigma circle (the training path); cull=False sums every splat at every pixel (exact,
    alpha mode only).  Returns [B,C,H,W] float32."""
    if cull:
        kw = dict(TILE=TILE, odds=odds, cutoff=cutoff)
        return _render(_lib.MODE_CULL, mu, log_scale, color, opacity, bg, H, W, theta, kw)
    if odds:
        raise NotImplementedError("odds compositing is only wired through the cull/octave path; "
                                  "use cull=True or render_alpha_octave")
    kw = dict(TILE=8, odds=False, cutoff=1e30)
    return _render(_lib.MODE_EXACT, mu, log_scale, color, opacity, bg, H, W, theta, kw)


def render_alpha_multires(mu, log_scale, color, opacity, bg, H, W, theta=None, n_coarse=None,
                          coarse_factor=8, cutoff=3.0, TILE=8, max_pairs=48_000_000, odds=False):
    """Coarse/fine split render (render_triton.py:879-922): the first n_coarse splats render at
    (H, W) / min(coarse_factor, max(1, min(H, W) // 8)), the rest at (H, W); raw sums are combined and
    composited once.  n_coarse=None renders everything at full resolution.  Returns [B,C,H,W]."""
    nc = -1 if n_coarse is None else int(n_coarse)
    kw = dict(TILE=TILE, odds=odds, cutoff=cutoff, n_coarse=nc, coarse_factor=coarse_factor, max_pairs=max_pairs)
    return _render(_lib.MODE_MULTIRES, mu, log_scale, color, opacity, bg, H, W, theta, kw)


def _octave_of(scale_px, base_texels=8.0, max_octaves=6):
    """Octave routing rule of render_triton.py:925-932 on a [B,N] pixel-scale tensor (host-side helper
    kept for API parity; the render kernels compute it on the device)."""
    o = torch.ceil(torch.log2((scale_px / base_texels).clamp_min(1e-6)))
    return o.clamp(0, max_octaves).to(torch.int64)


__all__ = ["PairBudgetExceeded", "render_alpha_octave", "render_alpha_full_triton", "render_alpha_multires",
           "activate_scale"]
