"""The reference's ``render`` module API (gaussian_splat_encoder/render.py) on the B200 kernels.

``render_alpha_full`` (render.py:90-110) is the exact every-pixel x every-splat alpha render; here it
runs the library's exact mode (GS_MODE_EXACT), the same kernels as ``render_alpha_full_triton(cull=False)``,
so no [B,P,N] tensor is materialised and ``chunk_pixels`` only exists for signature compatibility.
``render_alpha_subsampled`` (render.py:68-87) renders a pixel list through the library's point kernels
(gs_render_points_fwd / _bwd).
``gaussian_falloff`` / ``alpha_composite`` / ``_pixels`` are the reference's small tensor helpers
(render.py:34-65), kept as torch expressions for callers that use them directly.
"""

from __future__ import annotations

import torch

import ctypes as _C

from . import _lib
from .params import activate_scale  # noqa: F401


def gaussian_falloff(diff: torch.Tensor, scale: torch.Tensor, theta) -> torch.Tensor:
    """exp(-1/2 d^T Sigma^-1 d) per (pixel, splat); diff [B,P,N,2] (pixel - mu), scale [B,N,2], theta [B,N]
    or None (render.py:34-44)."""
    if theta is not None:
        cos_t, sin_t = torch.cos(theta), torch.sin(theta)
        dy, dx = diff[..., 0], diff[..., 1]
        rot_y = cos_t.unsqueeze(1) * dy + sin_t.unsqueeze(1) * dx
        rot_x = -sin_t.unsqueeze(1) * dy + cos_t.unsqueeze(1) * dx
        diff = torch.stack([rot_y, rot_x], dim=-1)
    maha = (diff.pow(2) / scale.unsqueeze(1).pow(2)).sum(-1)
    return torch.exp(-0.5 * maha)


def alpha_composite(falloff, opacity, color, bg):
    """Order-independent alpha blend of a materialised falloff [B,P,N] (render.py:47-58)."""
    alpha = (falloff * opacity.unsqueeze(1)).clamp(max=1.0 - 1e-4)
    T = torch.log1p(-alpha.float()).sum(-1).exp().to(alpha.dtype)
    asum = alpha.sum(-1).clamp_min(1e-8)
    fg = torch.bmm(alpha, color) / asum.unsqueeze(-1)
    return (1.0 - T).unsqueeze(-1) * fg + T.unsqueeze(-1) * bg.unsqueeze(1)


def _pixels(H, W, device, dtype):
    ys = torch.linspace(0.5 / H, 1 - 0.5 / H, H, device=device, dtype=dtype)
    xs = torch.linspace(0.5 / W, 1 - 0.5 / W, W, device=device, dtype=dtype)
    gy, gx = torch.meshgrid(ys, xs, indexing="ij")
    return torch.stack([gy, gx], dim=-1).reshape(H * W, 2)


def render_alpha_full(mu, log_scale, color, opacity, bg, H, W, theta=None, chunk_pixels=4096):
    """Exact full-resolution alpha render [B,C,H,W] (render.py:90-110), differentiable."""
    from .render_triton import render_alpha_full_triton

    return render_alpha_full_triton(mu, log_scale, color, opacity, bg, H, W, theta=theta, cull=False)


class _PointsRender(torch.autograd.Function):
    """All N splats composited (alpha mode) at a pixel list; the workspace of the forward carries the
    per-pixel sums into the backward."""

    @staticmethod
    def forward(ctx, mu, log_scale, color, opacity, bg, theta, px_idx, H, W):
        dev = _lib.require_cuda(mu, log_scale, color, opacity, bg, theta, px_idx)
        B, N, Cc = color.shape
        if mu.shape != (B, N, 2) or log_scale.shape != (B, N, 2) or opacity.shape != (B, N) or bg.shape[0] != B:
            raise ValueError("shape mismatch: mu/log_scale [B,N,2], color [B,N,C], opacity [B,N], bg [B,C]")
        if px_idx.dim() != 2 or px_idx.shape[0] != B:
            raise ValueError("pixel indices must be [B, n_px]")
        if not 1 <= Cc <= 3:
            raise ValueError(f"colour channels of one render call must be 1..3, got {Cc}")
        f = [None if t is None else t.detach().contiguous().float() for t in (mu, log_scale, color, opacity, bg, theta)]
        idx = px_idx.detach().contiguous().to(torch.int64)
        P = int(idx.shape[1])
        d = _lib.GsRenderDesc()
        d.mode, d.B, d.N, d.C, d.H, d.W = _lib.MODE_EXACT, B, N, Cc, int(H), int(W)
        d.tile, d.odds, d.has_theta, d.cutoff = 8, 0, int(theta is not None), 3.0
        with torch.cuda.device(dev):
            L = _lib.load()
            train = any(ctx.needs_input_grad[:6])
            nbytes = int(L.gs_render_points_workspace_size(_C.byref(d), P, int(train)))
            if nbytes == 0:
                raise ValueError("invalid render arguments")
            ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            out = torch.empty((B, Cc, P), dtype=torch.float32, device=dev)
            _lib.check(L.gs_render_points_fwd(_C.byref(d), P, _lib.ptr(idx), *[_lib.ptr(t) for t in f], _lib.ptr(out),
                                              _lib.ptr(ws), nbytes, _lib.stream_of(dev)), "gs_render_points_fwd")
        ctx.desc, ctx.P, ctx.ws = d, P, (ws if train else None)
        ctx.has_theta = theta is not None
        ctx.save_for_backward(f[0], f[1], f[2], f[3], f[4], f[5] if f[5] is not None else f[0].new_zeros(0), idx)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        mu, ls, col, op, bg, th, idx = ctx.saved_tensors
        th = th if ctx.has_theta else None
        dev = mu.device
        g = grad_out.contiguous().float()
        grads = [torch.empty_like(mu), torch.empty_like(ls), torch.empty_like(col), torch.empty_like(op),
                 torch.empty_like(bg), torch.empty_like(th) if th is not None else None]
        with torch.cuda.device(dev):
            L = _lib.load()
            ws = ctx.ws
            _lib.check(L.gs_render_points_bwd(_C.byref(ctx.desc), ctx.P, _lib.ptr(idx), _lib.ptr(ls), _lib.ptr(bg),
                                              _lib.ptr(th), _lib.ptr(g), *[_lib.ptr(x) for x in grads],
                                              _lib.ptr(ws), ws.numel(), _lib.stream_of(dev)), "gs_render_points_bwd")
        out = [gr if ctx.needs_input_grad[i] else None for i, gr in enumerate(grads)]
        return (*out, None, None, None)


def render_alpha_subsampled(mu, log_scale, color, opacity, bg, H, W, theta=None, n_pixels=10000,
                            pixel_indices=None):
    """Differentiable alpha-composited render at a subsample of pixels (render.py:68-87): every splat
    at every listed pixel.  pixel_indices [B, n_px] (flat y*W + x) or None for min(n_pixels, H*W)
    uniform draws per image (torch.randint on the splats' device, as the reference draws them).
    Returns (rendered [B,C,n_px], px_idx [B,n_px])."""
    B = color.shape[0]
    total = int(H) * int(W)
    if pixel_indices is not None:
        px_idx = pixel_indices
    else:
        px_idx = torch.randint(0, total, (B, min(int(n_pixels), total)), device=mu.device)
    C = color.shape[-1]
    if C <= 3:
        rendered = _PointsRender.apply(mu, log_scale, color, opacity, bg, theta, px_idx, int(H), int(W))
    else:  # groups of at most three channels composite independently (see render_triton._render)
        rendered = torch.cat([_PointsRender.apply(mu, log_scale, color[..., c:c + 3], opacity, bg[:, c:c + 3], theta,
                                                  px_idx, int(H), int(W)) for c in range(0, C, 3)], dim=1)
    return rendered, px_idx
