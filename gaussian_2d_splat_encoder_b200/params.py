"""Splat-parameter decode (reference: bigwolfeman/gaussian-2d-splat-encoder, gaussian_splat_encoder/params.py).

``SCALE_EPS``, ``activate_scale`` and ``assemble_gaussian_params`` keep the reference's names and
contract.  On CUDA tensors ``activate_scale`` runs the library's softplus kernel (gs_activate_scale) with
an autograd backward; on CPU tensors it evaluates the same formula with torch so consumers outside the
render path (statistics, descriptors) keep working.  The renderers never call it: their kernels apply
the same softplus on the device.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import _lib

# Floor width of the smallest splat in normalised units; part of the 9-vector contract (params.py:13-15).
SCALE_EPS = 1e-4


class _ActivateScale(torch.autograd.Function):
    @staticmethod
    def forward(ctx, log_scale):
        x = log_scale.detach().contiguous().float()
        out = torch.empty_like(x)
        with torch.cuda.device(x.device):
            _lib.check(_lib.load().gs_activate_scale(_lib.ptr(x), _lib.ptr(out), x.numel(),
                                                     _lib.stream_of(x.device)), "gs_activate_scale")
        ctx.save_for_backward(x)
        return out.to(log_scale.dtype)

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        d = torch.where(x > 20.0, torch.ones_like(x), torch.sigmoid(x))
        return g * d


def activate_scale(log_scale: torch.Tensor) -> torch.Tensor:
    """Raw log_scale channel -> the sigma every renderer draws with: softplus(log_scale) + SCALE_EPS
    (params.py:18-28)."""
    if log_scale.is_cuda:
        return _ActivateScale.apply(log_scale)
    return F.softplus(log_scale) + SCALE_EPS


def assemble_gaussian_params(enc_out: dict) -> torch.Tensor:
    """Encoder output dict -> [B, N, 9] = [mu(2), log_scale(2), theta(1), color(3), opacity(1)]
    (params.py:31-41); theta defaults to 0 and opacity to 1 when absent."""
    mu = enc_out["mu"]
    ls = enc_out["log_scale"]
    th = enc_out.get("theta")
    th = th.unsqueeze(-1) if th is not None else torch.zeros_like(mu[..., :1])
    col = enc_out["color"]
    op = enc_out.get("opacity")
    op = op.unsqueeze(-1) if op is not None else torch.ones_like(mu[..., :1])
    return torch.cat([mu, ls, th, col, op], dim=-1)
