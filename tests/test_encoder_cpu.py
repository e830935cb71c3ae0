"""Encoder host-side checks (no GPU): the fp32 oracle against the reference's own encoder outputs,
state-dict / random-init compatibility with the reference module, and the weight packing of the
first layer (7x7 stride 2 == 4x4 stride 1 on the space-to-depth input)."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from enc_util import GOLDEN_CFG, load_golden
from golden_util import GOLDEN


def test_random_init_matches_reference():
    """torch.manual_seed(0) + construction gives the reference's parameters (config 0)."""
    from gaussian_2d_splat_encoder_b200.efficient_encoder import EfficientGaussianEncoder

    d = np.load(GOLDEN / "encoder_cfg0.npz")
    torch.manual_seed(0)
    m = EfficientGaussianEncoder(**GOLDEN_CFG)
    sd = m.state_dict()
    assert sum(p.numel() for p in m.parameters()) == 833107
    for k, v in sd.items():
        got = np.array([v.double().sum().item(), v.double().square().sum().item(), v.flatten()[0].item()])
        assert np.allclose(got, d[f"p_{k}"], rtol=1e-12, atol=0), k


@pytest.mark.parametrize("name", ["encoder_cfg0", "encoder_golden64"])
def test_encoder_oracle_matches_reference(name):
    from gaussian_2d_splat_encoder_b200.efficient_encoder import EfficientGaussianEncoder
    from oracle import encoder_oracle as E

    d = np.load(GOLDEN / f"{name}.npz")
    if name == "encoder_cfg0":
        torch.manual_seed(0)
        sd = EfficientGaussianEncoder(**GOLDEN_CFG).state_dict()
    else:
        m = load_golden(EfficientGaussianEncoder)
        if m is None:
            pytest.skip("released checkpoint not available")
        sd = m.state_dict()
    o = E.encode(sd, GOLDEN_CFG, torch.from_numpy(d["image"]))
    for k in ("mu", "log_scale", "color", "opacity", "theta", "bg", "backbone_features"):
        assert np.abs(o[k].numpy() - d[k]).max() < 1e-5, k
    assert o["n_coarse"] == int(d["n_coarse"])


def test_first_layer_space_to_depth_packing():
    from gaussian_2d_splat_encoder_b200.efficient_encoder import pack_first_layer, space_to_depth_input

    g = torch.Generator().manual_seed(0)
    x = torch.randn(2, 4, 24, 40, generator=g, dtype=torch.float64)
    w = torch.randn(64, 4, 7, 7, generator=g, dtype=torch.float64)
    ref = F.conv2d(x, w, stride=2, padding=3)
    z = space_to_depth_input(x)                                 # [B, H/2, W/2, 16]
    wp = pack_first_layer(w).reshape(64, 4, 4, 16).permute(0, 3, 1, 2)   # [Co, 16, 4, 4]
    zin = F.pad(z.permute(0, 3, 1, 2), (2, 1, 2, 1))            # taps at offsets -2..+1
    out = F.conv2d(zin, wp)
    assert out.shape == ref.shape
    assert torch.allclose(out, ref, atol=1e-10, rtol=1e-10)


def test_pack_conv_order():
    from gaussian_2d_splat_encoder_b200.efficient_encoder import pack_conv

    w = torch.arange(2 * 3 * 3 * 3, dtype=torch.float32).reshape(2, 3, 3, 3)
    p = pack_conv(w)
    # K index = (kh*3 + kw)*Cin + c
    assert p[1, (2 * 3 + 1) * 3 + 2] == w[1, 2, 2, 1]


def test_golden_checkpoint_loads_strict():
    from gaussian_2d_splat_encoder_b200.efficient_encoder import EfficientGaussianEncoder

    m = load_golden(EfficientGaussianEncoder)
    if m is None:
        pytest.skip("released checkpoint not available")
    assert sum(p.numel() for p in m.parameters()) == 833107
