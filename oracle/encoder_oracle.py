"""TEST INFRASTRUCTURE ONLY: fp32 CPU restatement of the reference encoder's forward.

Restates EfficientGaussianEncoder.forward for variant 'adaptive' (bigwolfeman/gaussian-2d-splat-encoder,
gaussian_splat_encoder/efficient_encoder.py:306-378, with _Backbone :63-72, _UpBlock :89-91,
_SplatHead.forward :170-197, sobel_gradmag :123-130) as plain torch-CPU fp32 tensor math over a
state_dict, with the internal coarse render done by the C oracle (oracle/gsplat_oracle.c).  It is the
checker of the CUDA encoder and the CPU baseline of bench.py; the product never imports it.
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

from . import oracle as O


def _gelu_gn(x, sd, conv, gn):
    x = F.conv2d(x, sd[f"{conv}.weight"], sd[f"{conv}.bias"], stride=_STRIDES[conv], padding=_PADS[conv])
    x = F.gelu(x)
    return F.group_norm(x, 8, sd[f"{gn}.weight"], sd[f"{gn}.bias"], eps=1e-5)


_STRIDES = {"backbone.stage_s2.0": 2, "backbone.stage_s4.0": 2, "backbone.stage_s8.0": 2,
            "fine_decoder.blocks.0.fuse.0": 1}
_PADS = {"backbone.stage_s2.0": 3, "backbone.stage_s4.0": 1, "backbone.stage_s8.0": 1,
         "fine_decoder.blocks.0.fuse.0": 1}


def sobel_gradmag(img):
    gray = img.mean(1, keepdim=True)
    kx = torch.tensor([[-1, 0, 1], [-2, 0, 2], [-1, 0, 1]], dtype=img.dtype) / 4.0
    ky = kx.t().contiguous()
    gx = F.conv2d(gray, kx.view(1, 1, 3, 3), padding=1)
    gy = F.conv2d(gray, ky.view(1, 1, 3, 3), padding=1)
    return torch.sqrt(gx * gx + gy * gy + 1e-6)


def _head(feat, sd, name, M, offset_cells, use_rotation, min_opacity=0.0):
    B, _, fH, fW = feat.shape
    ys = torch.linspace(0.5 / fH, 1 - 0.5 / fH, fH)
    xs = torch.linspace(0.5 / fW, 1 - 0.5 / fW, fW)
    gy, gx = torch.meshgrid(ys, xs, indexing="ij")
    base = torch.stack([gy, gx], 0).unsqueeze(0).unsqueeze(0)
    off = offset_cells / max(fH, fW)

    def c1(k):
        return F.conv2d(feat, sd[f"{name}.{k}.weight"], sd[f"{name}.{k}.bias"])

    mu = base + torch.tanh(c1("mu_head").reshape(B, M, 2, fH, fW)) * off
    mu = mu.permute(0, 3, 4, 1, 2).reshape(B, fH * fW * M, 2).clamp(0.005, 0.995)
    ls = c1("scale_head").reshape(B, M, 2, fH, fW).permute(0, 3, 4, 1, 2).reshape(B, fH * fW * M, 2)
    col = torch.sigmoid(c1("color_head").reshape(B, M, 3, fH, fW).permute(0, 3, 4, 1, 2).reshape(B, -1, 3))
    op = torch.sigmoid(c1("opacity_head").reshape(B, M, fH, fW).permute(0, 2, 3, 1).reshape(B, fH * fW * M))
    if min_opacity > 0.0:
        op = min_opacity + (1.0 - min_opacity) * op
    th = None
    if use_rotation:
        th = torch.tanh(c1("theta_head").reshape(B, M, fH, fW).permute(0, 2, 3, 1).reshape(B, -1)) * (math.pi / 2)
    return dict(mu=mu, log_scale=ls, color=col, opacity=op, theta=th)


@torch.no_grad()
def encode(state_dict, cfg: dict, image: torch.Tensor) -> dict:
    """fp32 forward of the 'adaptive' encoder.  cfg: the constructor keywords of the checkpoint
    (gaussians_per_cell, fine_per_cell, residual_grid, coarse_min_scale, coarse_offset_cells,
    fine_offset_cells, coarse_min_opacity, use_rotation, odds)."""
    sd = {k: v.detach().float().cpu() for k, v in state_dict.items()}
    x = image.detach().float().cpu()
    M = cfg.get("gaussians_per_cell", 2)
    Mf = cfg.get("fine_per_cell", 2)
    rg = cfg.get("residual_grid", 64)
    use_rot = cfg.get("use_rotation", True)
    odds = cfg.get("odds", False)
    cms = cfg.get("coarse_min_scale", 0.04)
    floor = math.log(math.exp(cms) - 1.0) if cms > 0 else None
    grad = sobel_gradmag(x)
    xin = torch.cat([x, grad], 1)
    s2 = _gelu_gn(xin, sd, "backbone.stage_s2.0", "backbone.stage_s2.2")
    s4 = _gelu_gn(s2, sd, "backbone.stage_s4.0", "backbone.stage_s4.2")
    s8 = _gelu_gn(s4, sd, "backbone.stage_s8.0", "backbone.stage_s8.2")
    g8 = F.adaptive_avg_pool2d(grad, s8.shape[2:])
    fused = torch.cat([s8, g8], 1)
    bg = torch.sigmoid(F.linear(s8.mean(dim=(2, 3)), sd["bg_head.weight"], sd["bg_head.bias"]))
    coarse = _head(fused, sd, "coarse_head", M, cfg.get("coarse_offset_cells", 2.0), use_rot,
                   cfg.get("coarse_min_opacity", 0.0))
    if floor is not None:
        coarse["log_scale"] = coarse["log_scale"].clamp(min=floor)
    c = {k: (v.numpy() if v is not None else None) for k, v in coarse.items()}
    c_render = torch.from_numpy(O.render_alpha_octave(c["mu"], c["log_scale"], c["color"], c["opacity"],
                                                      bg.numpy(), rg, rg, theta=c["theta"], odds=odds))
    target_small = F.interpolate(x, size=(rg, rg), mode="bilinear", align_corners=False)
    resid = (target_small - c_render).abs()
    cond = torch.cat([resid, c_render.mean(1, keepdim=True)], 1)
    up = F.interpolate(s8, size=s4.shape[2:], mode="bilinear", align_corners=False)
    fine_feat = _gelu_gn(torch.cat([up, s4], 1), sd, "fine_decoder.blocks.0.fuse.0", "fine_decoder.blocks.0.fuse.2")
    ffH, ffW = fine_feat.shape[2:]
    cond_fine = F.interpolate(cond, size=(ffH, ffW), mode="bilinear", align_corners=False)
    g_fine = F.adaptive_avg_pool2d(grad, (ffH, ffW))
    fine = _head(torch.cat([fine_feat, g_fine, cond_fine], 1), sd, "fine_head", Mf, cfg.get("fine_offset_cells", 2.0),
                 use_rot)
    out = {k: torch.cat([coarse[k], fine[k]], 1) for k in ("mu", "log_scale", "color", "opacity")}
    out["theta"] = torch.cat([coarse["theta"], fine["theta"]], 1) if use_rot else None
    out["bg"] = bg
    out["n_gaussians"] = out["mu"].shape[1]
    out["n_coarse"] = coarse["mu"].shape[1]
    out["backbone_features"] = s8
    out["splat_features"] = fine_feat
    out["coarse_render"] = c_render
    return out


def psnr(a: np.ndarray, b: np.ndarray) -> float:
    mse = float(np.mean((np.asarray(a, np.float64) - np.asarray(b, np.float64)) ** 2))
    return -10.0 * math.log10(max(mse, 1e-12))
