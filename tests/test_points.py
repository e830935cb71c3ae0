"""Pixel-list render (render_alpha_subsampled, render.py:68-87): the float64 CPU oracle pinned against
fixtures the reference produced, and the CUDA point kernels (gs_render_points_fwd / _bwd, through the C
ABI) against the oracle.  Tolerances: rendered values 1e-4 absolute, splat gradients 1e-3 relative
(per-leaf max|diff| / max|ref|, the reference self-tests' metric)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from golden_util import GOLDEN, LEAVES, grad_rel

CASES = ("points_theta", "points_notheta")


def load(name):
    d = np.load(GOLDEN / f"{name}.npz", allow_pickle=False)
    ins = {n: d[f"in_{n}"] for n in LEAVES if f"in_{n}" in d.files}
    gC = torch.randn(d["out"].shape, generator=torch.Generator().manual_seed(int(d["gseed"]))).numpy()
    grads = {n: d[f"grad_{n}"] for n in LEAVES if f"grad_{n}" in d.files}
    return dict(H=int(d["H"]), W=int(d["W"]), ins=ins, idx=d["px_idx"], gC=gC, out=d["out"], grads=grads)


def oracle(ins, H, W, idx, gC):
    from oracle.points_oracle import render_points

    return render_points(ins["mu"], ins["log_scale"], ins["color"], ins["opacity"], ins["bg"], H, W, idx,
                         theta=ins.get("theta"), grad_out=gC)


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference(name):
    c = load(name)
    out, grads = oracle(c["ins"], c["H"], c["W"], c["idx"], c["gC"])
    assert np.abs(out - c["out"]).max() < 2e-6
    rel = grad_rel(grads, c["grads"])
    assert max(rel.values()) < 1e-4, rel


def _cuda_points(ins, H, W, idx, gC):
    from gaussian_2d_splat_encoder_b200.render import render_alpha_subsampled

    dev = torch.device("cuda")
    L = [torch.tensor(ins[n], device=dev, requires_grad=True) if n in ins else None for n in LEAVES]
    out, pidx = render_alpha_subsampled(*L[:5], H, W, theta=L[5], pixel_indices=torch.tensor(idx, device=dev))
    (out * torch.tensor(gC, device=dev)).sum().backward()
    grads = {n: t.grad.cpu().numpy() for n, t in zip(LEAVES, L) if t is not None}
    return out.detach().cpu().numpy(), grads, pidx


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_cuda_vs_oracle_golden(name):
    c = load(name)
    out, grads, _ = _cuda_points(c["ins"], c["H"], c["W"], c["idx"], c["gC"])
    ref_out, ref_grads = oracle(c["ins"], c["H"], c["W"], c["idx"], c["gC"])
    assert np.abs(out - ref_out).max() < 1e-4
    rel = grad_rel(grads, ref_grads)
    assert max(rel.values()) < 1e-3, rel


@pytest.mark.gpu
@pytest.mark.parametrize("B,N,H,W,P,theta", [(1, 4096, 256, 256, 2000, True), (2, 2500, 100, 77, 333, False),
                                             (1, 1, 16, 16, 1, True)])
def test_cuda_vs_oracle_sizes(B, N, H, W, P, theta):
    g = torch.Generator().manual_seed(B * 1000 + N)
    ins = dict(mu=torch.rand(B, N, 2, generator=g).numpy(),
               log_scale=(torch.randn(B, N, 2, generator=g) * 0.5 - 4.0).numpy(),
               color=torch.rand(B, N, 3, generator=g).numpy(),
               opacity=torch.sigmoid(torch.randn(B, N, generator=g) * 1.5 + 1.0).numpy(),
               bg=torch.rand(B, 3, generator=g).numpy())
    if theta:
        ins["theta"] = (torch.rand(B, N, generator=g) * 3.14159).numpy()
    idx = torch.randint(0, H * W, (B, P), generator=g).numpy()
    gC = torch.randn(B, 3, P, generator=g).numpy()
    out, grads, _ = _cuda_points(ins, H, W, idx, gC)
    ref_out, ref_grads = oracle(ins, H, W, idx, gC)
    assert np.abs(out - ref_out).max() < 1e-4
    rel = grad_rel(grads, ref_grads)
    assert max(rel.values()) < 1e-3, rel


@pytest.mark.gpu
def test_sampling_and_empty():
    from gaussian_2d_splat_encoder_b200.render import render_alpha_subsampled

    dev = torch.device("cuda")
    B, N = 2, 64
    mu = torch.rand(B, N, 2, device=dev)
    ls = torch.full((B, N, 2), -4.0, device=dev)
    col, op, bg = torch.rand(B, N, 3, device=dev), torch.rand(B, N, device=dev), torch.rand(B, 3, device=dev)
    out, idx = render_alpha_subsampled(mu, ls, col, op, bg, 20, 30, n_pixels=10000)
    assert out.shape == (B, 3, 600) and idx.shape == (B, 600)
    assert int(idx.min()) >= 0 and int(idx.max()) < 600
    # no splats: every pixel shows the background
    e = torch.zeros(B, 0, 2, device=dev)
    out0, _ = render_alpha_subsampled(e, e, torch.zeros(B, 0, 3, device=dev), torch.zeros(B, 0, device=dev), bg,
                                      20, 30, pixel_indices=idx[:, :50])
    assert torch.allclose(out0, bg.unsqueeze(-1).expand(B, 3, 50))
