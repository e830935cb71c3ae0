"""Seeded synthetic inputs for the benchmark configurations.

The reference ships no dataset for its hot path; its benchmark configurations are seeded synthetic
images and seeded splat sets.  These generators produce them with numpy / torch CPU generators so the
same seed yields the same bytes on every machine.

* ``synth_card``      - test-card image: mean of 3 linear colour gradients, filled axis-aligned
                        rectangles / ellipses of uniform colour, and 1-3 px strokes, clipped to [0,1]
                        (configs 0, 2, 3, 4).
* ``synth_splats_cfg1`` - the render-only splat set of config 1 (92,160 splats at 768x768).
"""

from __future__ import annotations

import math

import numpy as np
import torch


def synth_card(H: int, W: int, n_shapes: int = 40, n_strokes: int = 20, seed: int = 0) -> torch.Tensor:
    """Return a [1,3,H,W] float32 image in [0,1] drawn from ``np.random.PCG64(seed)``."""
    rng = np.random.Generator(np.random.PCG64(seed))
    yy, xx = np.meshgrid(np.arange(H, dtype=np.float64) + 0.5, np.arange(W, dtype=np.float64) + 0.5,
                         indexing="ij")
    yn, xn = yy / H, xx / W
    img = np.zeros((H, W, 3), dtype=np.float64)
    for _ in range(3):
        ang = rng.uniform(0.0, 2.0 * math.pi)
        c0 = rng.uniform(size=3)
        c1 = rng.uniform(size=3)
        t = np.cos(ang) * yn + np.sin(ang) * xn
        t = (t - t.min()) / max(t.max() - t.min(), 1e-12)
        img += (1.0 - t)[..., None] * c0 + t[..., None] * c1
    img /= 3.0
    def box(ylo, yhi, xlo, xhi):
        # pixel-centre window that holds every pixel a shape can cover (2 px margin); the per-pixel
        # tests below run on that window only and give the same mask as over the whole image
        r0, r1 = max(0, int(math.floor(ylo)) - 2), min(H, int(math.ceil(yhi)) + 2)
        c0, c1 = max(0, int(math.floor(xlo)) - 2), min(W, int(math.ceil(xhi)) + 2)
        return (slice(r0, max(r0, r1)), slice(c0, max(c0, c1)))

    for _ in range(n_shapes):
        kind = int(rng.integers(2))
        hh = rng.uniform(0.02, 0.25) * H
        ww = rng.uniform(0.02, 0.25) * W
        cy = rng.uniform(0.0, H)
        cx = rng.uniform(0.0, W)
        col = rng.uniform(size=3)
        win = box(cy - hh / 2, cy + hh / 2, cx - ww / 2, cx + ww / 2)
        y, x = yy[win], xx[win]
        if kind == 0:
            m = (np.abs(y - cy) <= hh / 2) & (np.abs(x - cx) <= ww / 2)
        else:
            m = ((y - cy) / (hh / 2)) ** 2 + ((x - cx) / (ww / 2)) ** 2 <= 1.0
        img[win][m] = col
    for _ in range(n_strokes):
        y0, y1 = rng.uniform(0.0, H, size=2)
        x0, x1 = rng.uniform(0.0, W, size=2)
        width = float(rng.integers(1, 4))
        col = rng.uniform(size=3)
        dy, dx = y1 - y0, x1 - x0
        L2 = max(dy * dy + dx * dx, 1e-12)
        r = width / 2.0
        # bands of 32 rows, each narrowed to the columns the segment (widened by r) can reach there
        for ya in range(max(0, int(min(y0, y1) - r) - 2), min(H, int(max(y0, y1) + r) + 3), 32):
            yb = ya + 32
            if abs(dy) > 1e-9:
                ta = min(max((ya - r - 2 - y0) / dy, 0.0), 1.0)
                tb = min(max((yb + r + 2 - y0) / dy, 0.0), 1.0)
                xa, xb = x0 + ta * dx, x0 + tb * dx
            else:
                xa, xb = x0, x1
            win = box(ya + 2, yb - 2, min(xa, xb) - r, max(xa, xb) + r)
            y, x = yy[win], xx[win]
            t = np.clip(((y - y0) * dy + (x - x0) * dx) / L2, 0.0, 1.0)
            d2 = (y - (y0 + t * dy)) ** 2 + (x - (x0 + t * dx)) ** 2
            img[win][d2 <= r ** 2] = col
    img = np.clip(img, 0.0, 1.0).astype(np.float32)
    return torch.from_numpy(np.ascontiguousarray(img.transpose(2, 0, 1)))[None]


def card_for_config(cfg: int, seed: int | None = None) -> torch.Tensor:
    """Images of the benchmark configurations: 0 -> 128^2 (40 shapes, 20 strokes, seed 0);
    2/3 -> 768^2 (500 shapes, 150 strokes; seed 2, or seeds 100-163 for config 3); 4 -> 2048^2."""
    if cfg == 0:
        return synth_card(128, 128, 40, 20, 0 if seed is None else seed)
    if cfg in (2, 3):
        return synth_card(768, 768, 500, 150, 2 if seed is None else seed)
    if cfg == 4:
        return synth_card(2048, 2048, 2000, 600, 4 if seed is None else seed)
    raise ValueError(f"no image for config {cfg}")


def synth_splats_cfg1(N: int = 92160, H: int = 768, W: int = 768, seed: int = 1):
    """Config-1 splat set (normalised (y,x) positions, pre-softplus log-scales, theta in [0,pi),
    colours and opacities in (0,1)), drawn from one CPU ``torch.Generator`` in a fixed order.
    sigma_px ~ exp(ln 2 + 0.4 N(0,1)) per axis; log_scale inverts ``softplus(ls) + 1e-4``."""
    g = torch.Generator().manual_seed(seed)
    mu = torch.rand(N, 2, generator=g)
    sig_px = torch.exp(math.log(2.0) + 0.4 * torch.randn(N, 2, generator=g))
    s = sig_px / float(min(H, W)) - 1e-4
    log_scale = torch.log(torch.expm1(s))
    theta = math.pi * torch.rand(N, generator=g)
    color = torch.rand(N, 3, generator=g)
    opacity = torch.sigmoid(1.0 + 1.5 * torch.randn(N, generator=g))
    bg = torch.rand(3, generator=g)
    target = torch.rand(3, H, W, generator=g)
    return dict(mu=mu[None], log_scale=log_scale[None], color=color[None], opacity=opacity[None],
                theta=theta[None], bg=bg[None], target=target[None])
