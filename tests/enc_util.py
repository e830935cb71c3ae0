"""Shared helpers of the encoder tests: the checkpoint config and where a local copy of the released
checkpoint may be found (it is never committed; tests that need it skip without it)."""

import inspect
import os
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]
CANDIDATES = [os.environ.get("GSPLAT_WEIGHTS", ""), str(ROOT / "weights" / "encoder_golden_d256.pt")]

# the released checkpoint's encoder configuration (its cfg['encoder'] minus image_size)
GOLDEN_CFG = dict(d_feature=256, stride=8, variant="adaptive", use_rotation=True, use_grad_input=True,
                  gaussians_per_cell=2, fine_per_cell=2, free_offset_cells=4.0, coarse_scale_bias=-3.1,
                  coarse_min_scale=0.04, fine_scale_bias=-5.0, free_scale_bias=-3.0, residual_grid=384,
                  norm_type="group", opacity_bias=0.0, fine_stride=4, odds=True)


def checkpoint_path():
    for c in CANDIDATES:
        if c and Path(c).exists():
            return Path(c)
    return None


def load_golden(cls):
    p = checkpoint_path()
    if p is None:
        return None
    ck = torch.load(p, map_location="cpu", weights_only=True)
    cfg = dict(ck["cfg"]["encoder"])
    accepted = set(inspect.signature(cls.__init__).parameters) - {"self"}
    unknown = set(cfg) - accepted - {"image_size"}
    assert not unknown, unknown
    m = cls(**{k: v for k, v in cfg.items() if k in accepted})
    m.load_state_dict(ck["model"], strict=True)
    return m.eval()
