"""TEST INFRASTRUCTURE ONLY: CPU restatement of the reference's pixel-list render
(bigwolfeman/gaussian-2d-splat-encoder, gaussian_splat_encoder/render.py:68-87, render_alpha_subsampled,
with gaussian_falloff render.py:34-44, alpha_composite render.py:47-65 and activate_scale
params.py:18-28), in float64 torch on the CPU, gradients by torch autograd of the same expressions.

Used as the checker of the CUDA point kernels (gs_render_points_fwd / _bwd) by the parity tests; the
product package never imports it.  Pinned against fixtures produced by the reference itself
(tests/golden/points_*.npz, written by tests/golden/make_golden.py).
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F


def _activate_scale(ls):
    """params.py:18-28: softplus (torch's threshold 20) + 1e-4."""
    return F.softplus(ls) + 1e-4


def composite_points(mu, ls, col, op, bg, theta, idx, H, W, chunk: int = 1 << 22):
    """The composite on torch tensors (autograd-capable, any dtype and channel count): every splat at
    every pixel of idx [B,P] (flat y*W + x); returns out [B,C,P]."""
    B, N, C = col.shape
    P = idx.shape[1]
    scale = _activate_scale(ls)
    py = ((idx // W).to(mu.dtype) + 0.5) / H
    px = ((idx % W).to(mu.dtype) + 0.5) / W
    pix = torch.stack([py, px], dim=-1)  # [B,P,2]
    # the [B,P,N] reductions of alpha_composite, chunked over pixels to bound memory
    step = max(1, chunk // max(N, 1))
    logT, asum, acol = [], [], []
    for p0 in range(0, P, step):
        d = pix[:, p0:p0 + step].unsqueeze(2) - mu.unsqueeze(1)  # [B,p,N,2]
        dy, dx = d[..., 0], d[..., 1]
        if theta is not None:
            c, s = torch.cos(theta).unsqueeze(1), torch.sin(theta).unsqueeze(1)
            dy, dx = c * dy + s * dx, -s * dy + c * dx
        maha = (dy / scale[..., 0].unsqueeze(1)) ** 2 + (dx / scale[..., 1].unsqueeze(1)) ** 2
        alpha = (torch.exp(-0.5 * maha) * op.unsqueeze(1)).clamp(max=1.0 - 1e-4)
        logT.append(torch.log1p(-alpha).sum(-1))
        asum.append(alpha.sum(-1))
        acol.append(torch.bmm(alpha, col))
    T = torch.exp(torch.cat(logT, 1))
    a = torch.cat(asum, 1).clamp_min(1e-8)
    fg = torch.cat(acol, 1) / a.unsqueeze(-1)
    return ((1.0 - T).unsqueeze(-1) * fg + T.unsqueeze(-1) * bg.unsqueeze(1)).permute(0, 2, 1)  # [B,C,P]


def render_points(mu, log_scale, color, opacity, bg, H, W, px_idx, theta=None, grad_out=None,
                  chunk: int = 1 << 22):
    """Every splat at every listed pixel.  Arrays in the reference layouts (mu [B,N,2] (y,x),
    log_scale [B,N,2] pre-softplus, color [B,N,C], opacity [B,N], bg [B,C], theta [B,N] or None,
    px_idx [B,P] flat y*W + x).  Returns out [B,C,P] (float64 numpy), and with grad_out [B,C,P] also the
    gradients of sum(out * grad_out) w.r.t. the leaves that were given (dict of float64 arrays)."""
    t = lambda a: None if a is None else torch.as_tensor(np.asarray(a), dtype=torch.float64)  # noqa: E731
    leaves = [t(mu), t(log_scale), t(color), t(opacity), t(bg), t(theta)]
    need = grad_out is not None
    if need:
        for x in leaves:
            if x is not None:
                x.requires_grad_(True)
    mu_, ls_, col_, op_, bg_, th_ = leaves
    idx = torch.as_tensor(np.asarray(px_idx), dtype=torch.int64)
    out = composite_points(mu_, ls_, col_, op_, bg_, th_, idx, H, W, chunk)
    if not need:
        return out.detach().numpy()
    g = torch.as_tensor(np.asarray(grad_out), dtype=torch.float64)
    (out * g).sum().backward()
    names = ("mu", "log_scale", "color", "opacity", "bg", "theta")
    grads = {n: x.grad.numpy() for n, x in zip(names, leaves) if x is not None}
    return out.detach().numpy(), grads
