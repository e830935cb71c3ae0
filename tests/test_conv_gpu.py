"""tcgen05 implicit-GEMM convolution (gs_conv2d, through the C ABI) against torch's fp32 convolution of
the same bf16-rounded operands: bias + exact GELU fused, GroupNorm(8) partial sums accumulated."""

import ctypes as C

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


class ConvDesc(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("B", "H", "W", "Cin", "Cout", "kh", "kw", "stride", "pad", "Ho", "Wo",
                                         "gelu", "kind")]


def run_conv(lib, x_nhwc, w_packed, bias, Cout, kh, kw, stride, pad, Ho=0, Wo=0, gelu=1, kind=0):
    from gaussian_2d_splat_encoder_b200 import _lib

    B, H, W, Ci = x_nhwc.shape
    d = ConvDesc(B, H, W, Ci, Cout, kh, kw, stride, pad, Ho, Wo, gelu, kind)
    Ho_ = Ho or (H + 2 * pad - kh) // stride + 1
    Wo_ = Wo or (W + 2 * pad - kw) // stride + 1
    out = torch.empty(B, Ho_, Wo_, Cout, dtype=torch.bfloat16, device="cuda")
    stats = torch.zeros(B, 8, 2, dtype=torch.float64, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = lib.gs_conv2d(C.byref(d), _lib.ptr(x_nhwc), _lib.ptr(w_packed), _lib.ptr(bias), _lib.ptr(out),
                       _lib.ptr(stats), _lib.ptr(err), _lib.stream_of(torch.device("cuda")))
    torch.cuda.synchronize()
    assert st == 0
    assert int(err.item()) == 0, "a bounded device wait gave up"
    return out, stats


def check(out, ref, stats):
    ref_nhwc = ref.permute(0, 2, 3, 1)
    o = out.float()
    err = (o - ref_nhwc).abs()
    tol = 8e-3 * ref_nhwc.abs() + 2e-3 * ref_nhwc.abs().max()
    assert bool((err <= tol).all()), f"max err {err.max().item():.3e} (ref max {ref_nhwc.abs().max().item():.3e})"
    B, Co = ref.shape[0], ref.shape[1]
    g = ref.double().reshape(B, 8, Co // 8, -1)
    s = torch.stack([g.sum((2, 3)), g.square().sum((2, 3))], -1)
    assert torch.allclose(stats, s, rtol=2e-3, atol=1e-2 * float(s.abs().max())), (stats - s).abs().max()


def _rand(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, generator=g, device="cuda") * scale)


@pytest.mark.parametrize("shape", [(2, 64, 64), (1, 48, 80), (1, 768, 768), (2, 256, 512), (1, 202, 256)])
def test_first_layer(lib, shape):
    from gaussian_2d_splat_encoder_b200.efficient_encoder import pack_first_layer, space_to_depth_input

    B, H, W = shape
    x = _rand(B, 4, H, W).bfloat16()
    w = _rand(64, 4, 7, 7, scale=0.1, seed=1).bfloat16()
    b = _rand(64, scale=0.1, seed=2)
    z = space_to_depth_input(x)
    wp = pack_first_layer(w.float()).bfloat16().contiguous()
    out, st = run_conv(lib, z, wp, b, 64, 4, 4, 1, 2, Ho=H // 2, Wo=W // 2, kind=1)
    ref = F.gelu(F.conv2d(x.float(), w.float(), b, stride=2, padding=3))
    check(out, ref, st)


@pytest.mark.parametrize("shape", [(1, 768, 768), (2, 256, 512)])
def test_first_layer_halo_matches_per_tap_loads(lib, shape, monkeypatch):
    """The halo form of the first layer (one window per item, taps as offset views, unswizzled) issues the
    same MMAs on the same operands as the per-tap TMA form (GS_CONV_HALO=0): identical outputs."""
    from gaussian_2d_splat_encoder_b200.efficient_encoder import pack_first_layer, space_to_depth_input

    B, H, W = shape
    x = _rand(B, 4, H, W, seed=5).bfloat16()
    w = _rand(64, 4, 7, 7, scale=0.1, seed=6).bfloat16()
    b = _rand(64, scale=0.1, seed=7)
    z = space_to_depth_input(x)
    wp = pack_first_layer(w.float()).bfloat16().contiguous()
    outs = []
    for flag in ("1", "0"):
        monkeypatch.setenv("GS_CONV_HALO", flag)
        out, _ = run_conv(lib, z, wp, b, 64, 4, 4, 1, 2, Ho=H // 2, Wo=W // 2, kind=1)
        outs.append(out.clone())
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]), (outs[0].float() - outs[1].float()).abs().max()


@pytest.mark.parametrize("Ci,Co,H,W,stride,nb", [(64, 128, 32, 48, 2, 2), (128, 256, 16, 24, 2, 2),
                                                 (384, 128, 16, 24, 1, 2), (64, 128, 384, 384, 2, 2),
                                                 (128, 256, 192, 192, 2, 2), (384, 128, 192, 192, 1, 2),
                                                 (64, 64, 20, 36, 1, 2), (64, 128, 384, 384, 2, 4),
                                                 (384, 128, 192, 192, 1, 4), (128, 256, 192, 192, 2, 4)])
def test_conv3x3(lib, Ci, Co, H, W, stride, nb):
    """nb = 4: the shapes of the batched throughput form."""
    from gaussian_2d_splat_encoder_b200.efficient_encoder import pack_conv

    x = _rand(nb, Ci, H, W, seed=3).bfloat16()
    w = _rand(Co, Ci, 3, 3, scale=(1.0 / (9 * Ci)) ** 0.5, seed=4).bfloat16()
    b = _rand(Co, scale=0.1, seed=5)
    xn = x.permute(0, 2, 3, 1).contiguous()
    out, st = run_conv(lib, xn, pack_conv(w).contiguous(), b, Co, 3, 3, stride, 1)
    ref = F.gelu(F.conv2d(x.float(), w.float(), b, stride=stride, padding=1))
    check(out, ref, st)
