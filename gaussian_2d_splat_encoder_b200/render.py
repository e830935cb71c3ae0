"""The reference's ``render`` module API (gaussian_splat_encoder/render.py) on the B200 kernels.

``render_alpha_full`` (render.py:90-110) is the exact every-pixel x every-splat alpha render; here it
runs the library's exact mode (GS_MODE_EXACT), the same kernels as ``render_alpha_full_triton(cull=False)``,
so no [B,P,N] tensor is materialised and ``chunk_pixels`` only exists for signature compatibility.
``gaussian_falloff`` / ``alpha_composite`` / ``_pixels`` are the reference's small tensor helpers
(render.py:34-65), kept as torch expressions for callers that use them directly.
"""

from __future__ import annotations

import torch

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
