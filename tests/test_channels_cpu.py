"""More than three colour channels: the render entry points split them into groups of at most three,
render each group with one library call and concatenate.  Checked on the CPU with the library call
replaced by the float64 oracle composite (the same math), so the test covers the grouping itself: channel
order, background slices, and the shared leaves' gradients summed over the groups."""

import pytest
import torch

from oracle import points_oracle as PO


def _leaves(B, N, C, seed=0):
    g = torch.Generator().manual_seed(seed)
    t = lambda *s: torch.rand(*s, generator=g, dtype=torch.float64)  # noqa: E731
    return [t(B, N, 2), t(B, N, 2) - 3.0, t(B, N, C), t(B, N) * 0.9, t(B, C), t(B, N) * 3.0]


def _grads(out, leaves, seed=1):
    gC = torch.randn(out.shape, generator=torch.Generator().manual_seed(seed), dtype=torch.float64)
    for x in leaves:
        x.grad = None
    (out * gC).sum().backward()
    return [x.grad.clone() for x in leaves]


def _check(fn_ours, fn_ref, B=2, N=40, C=5):
    a = [x.requires_grad_(True) for x in _leaves(B, N, C)]
    out = fn_ours(a)
    ga = _grads(out, a)
    b = [x.detach().clone().requires_grad_(True) for x in a]
    ref = fn_ref(b)
    gb = _grads(ref, b)
    assert out.shape == ref.shape
    assert torch.allclose(out, ref, rtol=0, atol=1e-12)
    for x, y in zip(ga, gb):
        assert torch.allclose(x, y, rtol=1e-10, atol=1e-13)


@pytest.mark.parametrize("C", [4, 5, 7])
def test_subsampled_channel_groups(monkeypatch, C):
    from gaussian_2d_splat_encoder_b200 import render as R

    widths = []

    class OracleCall:
        @staticmethod
        def apply(mu, ls, col, op, bg, th, idx, H, W):
            widths.append(col.shape[-1])
            return PO.composite_points(mu, ls, col, op, bg, th, idx, H, W)

    monkeypatch.setattr(R, "_PointsRender", OracleCall)
    H, W = 12, 10
    idx = torch.randint(0, H * W, (2, 37), generator=torch.Generator().manual_seed(3))
    _check(lambda L: R.render_alpha_subsampled(*L[:5], H, W, theta=L[5], pixel_indices=idx)[0],
           lambda L: PO.composite_points(*L[:5], L[5], idx, H, W), C=C)
    assert widths == [min(3, C - c) for c in range(0, C, 3)]


@pytest.mark.parametrize("C", [4, 6])
def test_full_render_channel_groups(monkeypatch, C):
    from gaussian_2d_splat_encoder_b200 import render_triton as rt

    H, W = 9, 11
    every = torch.arange(H * W).expand(2, H * W)

    class OracleCall:
        @staticmethod
        def apply(mu, ls, col, op, bg, th, cfg):
            assert col.shape[-1] <= 3 and cfg[1:3] == (H, W)
            out = PO.composite_points(mu, ls, col, op, bg, th, every, H, W)
            return out.reshape(out.shape[0], out.shape[1], H, W)

    monkeypatch.setattr(rt, "_Render", OracleCall)
    _check(lambda L: rt.render_alpha_full_triton(*L[:5], H, W, theta=L[5]),
           lambda L: PO.composite_points(*L[:5], L[5], every, H, W).reshape(2, C, H, W), C=C)


def test_three_channels_take_one_call(monkeypatch):
    from gaussian_2d_splat_encoder_b200 import render_triton as rt

    calls = []

    class OracleCall:
        @staticmethod
        def apply(mu, ls, col, op, bg, th, cfg):
            calls.append(col.shape[-1])
            return torch.zeros(col.shape[0], col.shape[-1], cfg[1], cfg[2], dtype=col.dtype)

    monkeypatch.setattr(rt, "_Render", OracleCall)
    L = _leaves(1, 5, 3)
    rt.render_alpha_octave(*L[:5], 8, 8, theta=L[5])
    assert calls == [3]
